// Sparse spin block kernel on bit-packed state.
//
// State layout: row r holds n_chains bits in words [r][n_chains/32]; bit c of
// the row (word c/32, bit c%32) is 1 when chain c's spin is -1.  One row of 256
// chains is 32 bytes, so the state of a million-node graph (32 MiB at 256
// chains) stays resident in L2 and a neighbour fetch is a single sector.
//
// Work item = (row, slice of 256 chains); one warp per item, lane l owns
// chains 8l..8l+7 of the slice, i.e. byte l of the slice's 32 bytes.  Each warp
// keeps two items in flight: the neighbour rows of item i+1 are staged into
// shared memory with cp.async (8 lanes x 4 bytes per row) while item i is
// computed, and the CSR metadata of item i+2 is fetched meanwhile.
//
// Field: for rows with d >= 5 neighbours the warp writes the 2^t (t = min(d, 8))
// left-to-right float32 partial sums of +-w_0..+-w_(t-1) into shared memory
// (entry bit k set = spin k is -1); each lane gathers its byte of the first t
// neighbour rows, transposes the 8x8 bit block so that byte v holds chain v's
// sign bits, and reads chain v's field with one lookup.  Remaining neighbours
// are added afterwards in CSR order with the sign flip of their weight, so the
// field is bit-identical to the sequential float32 sum of w*s
// (tt_thrml/compiler.py:303-318).  RNG words follow the same chain -> Philox
// counter mapping as the int8 kernel, so both layouts draw identical samples.
#include "spin_common.cuh"

#ifndef TTHRML_BITS_MIN_BLOCKS
#define TTHRML_BITS_MIN_BLOCKS 5
#endif
#ifndef TTHRML_BITS_STAGE_ROWS
#define TTHRML_BITS_STAGE_ROWS 16
#endif

namespace tthrml {
namespace {

constexpr int kBitsThreads = 128;
constexpr int kBitsStageRows = TTHRML_BITS_STAGE_ROWS;
constexpr int kSliceBytes = 32;  // 256 chains

// Stages the first kBitsStageRows neighbour rows of an item (32 bytes each):
// lane l copies half (l & 1) of neighbour row (l >> 1) with one 16-byte copy.
static_assert(kBitsStageRows == 16, "one 16-byte copy per lane stages 16 rows of 32 bytes");
__device__ __forceinline__ void issue_rows_bits(const RowInfo& m, int64_t word0, bool valid, const uint32_t* state,
                                                int64_t W, unsigned char* stage_buf, int lane) {
  if (!valid) return;
  const int staged = m.deg < kBitsStageRows ? m.deg : kBitsStageRows;
  const int k = lane >> 1, half = lane & 1;
  const int32_t j = __shfl_sync(0xffffffffu, m.col, k);
  if (k < staged) cp_async_bytes<16>(stage_buf + k * kSliceBytes + half * 16, state + (int64_t)j * W + word0 + half * 4);
}

// acc[v] += w * s_v for the 8 chains of one lane, s_v = -1 where bit v of b is set.
__device__ __forceinline__ void accumulate_bits(float (&acc)[8], uint32_t b, float w) {
  const uint32_t wb = __float_as_uint(w);
#pragma unroll
  for (int v = 0; v < 8; ++v) acc[v] = __fadd_rn(acc[v], __uint_as_float(wb ^ ((b << (31 - v)) & 0x80000000u)));
}

template <bool VARIATES>
__global__ void __launch_bounds__(kBitsThreads, TTHRML_BITS_MIN_BLOCKS) k_spin_bits(
    const int64_t* __restrict__ row_ptr, const int32_t* __restrict__ cols, const float* __restrict__ vals,
    const float* __restrict__ bias, int64_t row_start, int64_t n_rows, uint32_t* state, int64_t W,
    int64_t chain_offset, const float* __restrict__ variates, int64_t variates_sweeps, uint64_t seed,
    uint32_t sweep_base, const tthrml_run_ctl* __restrict__ ctl) {
  extern __shared__ __align__(16) unsigned char smem[];
  constexpr int kStageBytes = kBitsStageRows * kSliceBytes;
  constexpr int kWarpBytes = 2 * kStageBytes + (1 << kTableBits) * 4;
  const int lane = threadIdx.x & 31;
  unsigned char* wbuf = smem + (size_t)(threadIdx.x >> 5) * kWarpBytes;
  float* table = reinterpret_cast<float*>(wbuf + 2 * kStageBytes);
  const int64_t C = W * 32;
  const int64_t slices = W / 8;
  const int64_t items = n_rows * slices;
  const int64_t stride = ((int64_t)gridDim.x * blockDim.x) >> 5;
  int64_t item = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t sweep = sweep_base + (ctl ? ctl->sweep : 0u);
  const uint64_t sd = ctl ? ctl->seed : seed;
  const PhiloxKeys keys = philox_keys(seed_lo(sd), seed_hi(sd));
  const unsigned char* state_bytes = reinterpret_cast<const unsigned char*>(state);
  auto row_of = [&](int64_t it) -> int64_t { return slices == 1 ? it : (int64_t)((uint64_t)it / (uint64_t)slices); };

  RowInfo cur{}, nxt{};
  load_row(row_of(item), n_rows, row_ptr, cols, vals, bias, lane, cur);
  int stage = 0;
  issue_rows_bits(cur, (item - cur.r * slices) * 8, item < items, state, W, wbuf, lane);
  cp_async_commit();
  int64_t next = item + stride;
  if (next < items) load_row(row_of(next), n_rows, row_ptr, cols, vals, bias, lane, nxt);

  while (item < items) {
    issue_rows_bits(nxt, (next - nxt.r * slices) * 8, next < items, state, W, wbuf + (stage ^ 1) * kStageBytes, lane);
    cp_async_commit();
    RowInfo after{};
    if (next + stride < items) load_row(row_of(next + stride), n_rows, row_ptr, cols, vals, bias, lane, after);

    const int64_t slice = item - cur.r * slices;
    const int64_t c0 = slice * 256 + lane * 8;        // first chain of this lane
    const int64_t byte0 = slice * kSliceBytes + lane;  // this lane's byte within a row
    const int64_t row = row_start + cur.r;
    uint32_t bits[8];
    if (!VARIATES) {  // independent of the neighbour data: computed while it is in flight
      const int64_t g0 = chain_offset + c0;
#pragma unroll
      for (int v = 0; v < 8; v += 4) {
        const u32x4 rr = philox4x32_10(u32x4{(uint32_t)((g0 + v) >> 2), (uint32_t)row, sweep, kSaltSpin}, keys);
        bits[v] = rr.x;
        bits[v + 1] = rr.y;
        bits[v + 2] = rr.z;
        bits[v + 3] = rr.w;
      }
    }

    const int deg = cur.deg;
    const int staged = deg < kBitsStageRows ? deg : kBitsStageRows;
    const unsigned char* sbuf = wbuf + stage * kStageBytes + lane;
    float acc[8];
    int done = 0;
    if (deg >= 5) {
      const int t = deg < kTableBits ? deg : kTableBits;
      __syncwarp();  // the previous item's lookups are finished before the table is rewritten
      build_table(table, cur.w, t, lane);
      cp_async_wait<1>();
      __syncwarp();  // table and this item's staged rows are visible to the warp
      uint32_t lo = 0u, hi = 0u;
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (k < t) lo |= (uint32_t)sbuf[k * kSliceBytes] << (8 * k);
#pragma unroll
      for (int k = 4; k < 8; ++k)
        if (k < t) hi |= (uint32_t)sbuf[k * kSliceBytes] << (8 * (k - 4));
      transpose8x8(lo, hi);  // byte v = sign bits of chain v over neighbours 0..7
#pragma unroll
      for (int v = 0; v < 4; ++v) acc[v] = table[(lo >> (8 * v)) & 0xFFu];
#pragma unroll
      for (int v = 0; v < 4; ++v) acc[v + 4] = table[(hi >> (8 * v)) & 0xFFu];
      done = t;
    } else {
#pragma unroll
      for (int v = 0; v < 8; ++v) acc[v] = 0.0f;
      cp_async_wait<1>();
      __syncwarp();
    }
    for (int k = done; k < staged; ++k) {
      const float w = __shfl_sync(0xffffffffu, cur.w, k);
      accumulate_bits(acc, sbuf[k * kSliceBytes], w);
    }
    // neighbours kBitsStageRows..31: columns in registers, bytes read directly
    const int first_chunk = deg < 32 ? deg : 32;
    for (int k = kBitsStageRows; k < first_chunk; ++k) {
      const int32_t j = __shfl_sync(0xffffffffu, cur.col, k);
      const float w = __shfl_sync(0xffffffffu, cur.w, k);
      accumulate_bits(acc, state_bytes[(int64_t)j * W * 4 + byte0], w);
    }
    for (int64_t eb = cur.e0 + 32; eb < cur.e0 + deg; eb += 32) {  // more than 32 neighbours
      const int n = (int)min((int64_t)32, cur.e0 + deg - eb);
      const int32_t my_col = lane < n ? __ldg(cols + eb + lane) : 0;
      const float my_w = lane < n ? __ldg(vals + eb + lane) : 0.0f;
      for (int k = 0; k < n; ++k) {
        const int32_t j = __shfl_sync(0xffffffffu, my_col, k);
        const float w = __shfl_sync(0xffffffffu, my_w, k);
        accumulate_bits(acc, state_bytes[(int64_t)j * W * 4 + byte0], w);
      }
    }

    uint32_t down = 0u;  // bit v set = chain v samples -1
    if (VARIATES) {
      // the host never runs past variates_sweeps; the modulo keeps misuse in bounds
      const int64_t vs = (int64_t)(sweep % (uint32_t)(variates_sweeps > 0 ? variates_sweeps : 1));
      const float* lrow = variates + (vs * n_rows + cur.r) * C + c0;
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const float gamma = bias ? __fadd_rn(cur.b, acc[v]) : acc[v];
        down |= (__fmul_rn(2.0f, gamma) > __ldg(lrow + v) ? 0u : 1u) << v;
      }
    } else {
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const float gamma = bias ? __fadd_rn(cur.b, acc[v]) : acc[v];
        down |= (spin_up_fast(gamma, bits[v]) ? 0u : 1u) << v;
      }
    }
    reinterpret_cast<unsigned char*>(state)[row * W * 4 + byte0] = (unsigned char)down;

    __syncwarp();  // every lane is done with this stage before it is refilled
    stage ^= 1;
    cur = nxt;
    nxt = after;
    item = next;
    next += stride;
  }
  cp_async_wait<0>();
}

template <bool VARIATES>
int launch_bits(const int64_t* rp, const int32_t* cols, const float* vals, const float* bias, int64_t row_start,
                int64_t n_rows, uint32_t* state, int64_t W, int64_t chain_offset, const float* variates,
                int64_t variates_sweeps, uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl, cudaStream_t s) {
  constexpr int smem = (kBitsThreads / 32) * (2 * kBitsStageRows * kSliceBytes + (1 << kTableBits) * 4);
  static int per_sm = 0, sms = 0;  // same values from every thread: a benign race
  if (!per_sm) {
    int dev = 0, n = 0, b = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_spin_bits<VARIATES>, kBitsThreads, smem);
    if (e != cudaSuccess) return cuda_status(e, "k_spin_bits set-up");
    sms = n;
    per_sm = b > 0 ? b : 1;
  }
  const int64_t items = n_rows * (W / 8);
  const int64_t need = (items + kBitsThreads / 32 - 1) / (kBitsThreads / 32);
  const int64_t full = (int64_t)sms * per_sm;
  const int grid = (int)(need < full ? (need > 0 ? need : 1) : full);
  k_spin_bits<VARIATES><<<grid, kBitsThreads, smem, s>>>(rp, cols, vals, bias, row_start, n_rows, state, W,
                                                        chain_offset, variates, variates_sweeps, seed, sweep, ctl);
  return launch_status("k_spin_bits launch");
}

}  // namespace

// 16 chains per lane (spin_bits16.cu)
template <bool VARIATES>
int launch_bits16(const int64_t* rp, const int32_t* cols, const float* vals, const float* bias, int64_t row_start,
                  int64_t n_rows, uint32_t* state, int64_t W, int64_t chain_offset, const float* variates,
                  int64_t variates_sweeps, uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl,
                  const int32_t* row_order, cudaStream_t s);

}  // namespace tthrml

#ifndef TTHRML_BITS16
#define TTHRML_BITS16 1
#endif

namespace {
int spin_bits_step(const int64_t* row_ptr, const int32_t* cols, const float* vals, const float* bias,
                   int64_t row_start, int64_t n_rows, uint32_t* state, int64_t n_chains, int64_t chain_offset,
                   const float* variates, int64_t variates_sweeps, uint64_t seed, uint32_t sweep,
                   const tthrml_run_ctl* ctl, const int32_t* row_order, void* stream) {
  using namespace tthrml;
  if (n_rows == 0) return TTHRML_OK;
  if (!row_ptr || !cols || !vals || !state || n_rows < 0 || row_start < 0) {
    set_error("tthrml_spin_bits_step: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  if (n_chains <= 0 || n_chains % 256 || chain_offset % 4) {
    set_error("tthrml_spin_bits_step: n_chains must be a positive multiple of 256 and chain_offset a multiple of 4 "
              "(got %lld, %lld)", (long long)n_chains, (long long)chain_offset);
    return TTHRML_ERR_ARG;
  }
  if (((uintptr_t)state) % 16) {
    set_error("tthrml_spin_bits_step: state must be 16-byte aligned");
    return TTHRML_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t W = n_chains / 32;
  if (TTHRML_BITS16) {
    if (variates)
      return launch_bits16<true>(row_ptr, cols, vals, bias, row_start, n_rows, state, W, chain_offset, variates,
                                 variates_sweeps, seed, sweep, ctl, row_order, s);
    return launch_bits16<false>(row_ptr, cols, vals, bias, row_start, n_rows, state, W, chain_offset, variates,
                                variates_sweeps, seed, sweep, ctl, row_order, s);
  }
  if (variates)
    return launch_bits<true>(row_ptr, cols, vals, bias, row_start, n_rows, state, W, chain_offset, variates,
                             variates_sweeps, seed, sweep, ctl, s);
  return launch_bits<false>(row_ptr, cols, vals, bias, row_start, n_rows, state, W, chain_offset, variates,
                            variates_sweeps, seed, sweep, ctl, s);
}
}  // namespace

extern "C" int tthrml_spin_bits_step(const int64_t* row_ptr, const int32_t* cols, const float* vals,
                                     const float* bias, int64_t row_start, int64_t n_rows, uint32_t* state,
                                     int64_t n_chains, int64_t chain_offset, const float* variates,
                                     int64_t variates_sweeps, uint64_t seed, uint32_t sweep,
                                     const tthrml_run_ctl* ctl, void* stream) {
  return spin_bits_step(row_ptr, cols, vals, bias, row_start, n_rows, state, n_chains, chain_offset, variates,
                        variates_sweeps, seed, sweep, ctl, nullptr, stream);
}

extern "C" int tthrml_spin_bits_step_ordered(const int64_t* row_ptr, const int32_t* cols, const float* vals,
                                             const float* bias, int64_t row_start, int64_t n_rows, uint32_t* state,
                                             int64_t n_chains, int64_t chain_offset, const float* variates,
                                             int64_t variates_sweeps, uint64_t seed, uint32_t sweep,
                                             const tthrml_run_ctl* ctl, const int32_t* row_order, void* stream) {
  if (!row_order) {
    tthrml::set_error("tthrml_spin_bits_step_ordered: NULL row order");
    return TTHRML_ERR_ARG;
  }
  return spin_bits_step(row_ptr, cols, vals, bias, row_start, n_rows, state, n_chains, chain_offset, variates,
                        variates_sweeps, seed, sweep, ctl, row_order, stream);
}
