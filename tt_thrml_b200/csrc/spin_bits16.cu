// Sparse spin block kernel on bit-packed state, 16 chains per lane.
//
// Same state layout, arithmetic and Philox stream as the 8-chain kernel of
// spin_bits.cu, with the work item (row, slice of 256 chains) given to a
// half-warp: lane h of a half owns chains 16h..16h+15 of the slice, i.e. bytes
// 2h, 2h+1 of the slice's 32 bytes.  A warp therefore carries two items at a
// time and every per-row cost -- row metadata, staging copies, the
// partial-sum table, loop control -- is spread over 16 chains per lane
// instead of 8.
//
// Per item: the first 16 neighbour rows are staged into shared memory with two
// 16-byte cp.async per lane (double-buffered: the next item's rows arrive
// while this one computes); the half-warp writes the 256 left-to-right
// float32 partial sums of +-w_0..+-w_7 (weights past the degree are zero,
// which adds exact zeros) and each lane gathers its two bytes of the first
// eight neighbour rows, transposes them into one 8-bit index per chain and
// reads the chain's field with one lookup; neighbours 8 and up are added in
// CSR order.  The field is therefore the sequential float32 sum of w*s
// (tt_thrml/compiler.py:303-318), bit for bit.  Every shuffle runs on the full
// warp with loop bounds made uniform over the two halves.
#include "spin_common.cuh"

#ifndef TTHRML_BITS16_MIN_BLOCKS
#define TTHRML_BITS16_MIN_BLOCKS 3
#endif

namespace tthrml {
namespace {

constexpr int kB16Threads = 128;
constexpr int kB16StageRows = 16;
constexpr int kB16Slice = 32;                               // bytes of one row slice (256 chains)
constexpr int kB16StageBytes = kB16StageRows * kB16Slice;   // one item's staged rows
constexpr int kB16HalfBytes = 2 * kB16StageBytes + 256 * 4; // two stages + the partial-sum table
constexpr unsigned kFull = 0xffffffffu;

struct Row16 {
  int64_t r;    // block-local row
  int64_t e0;   // first term
  int32_t deg;
  int32_t col;  // lane h of the half holds column h (h < 16)
  float w;      // lane h holds weight h (0 past the degree)
  float b;
};

__device__ __forceinline__ void load_row16(int64_t r, bool valid, const int64_t* __restrict__ rp,
                                           const int32_t* __restrict__ cols, const float* __restrict__ vals,
                                           const float* __restrict__ bias, int lh, Row16& m) {
  m.r = r;
  m.e0 = 0;
  m.deg = 0;
  m.col = 0;
  m.w = 0.0f;
  m.b = 0.0f;
  if (!valid) return;
  m.e0 = __ldg(rp + r);
  m.deg = (int)(__ldg(rp + r + 1) - m.e0);
  const int n = m.deg < 16 ? m.deg : 16;
  if (lh < n) {
    m.col = __ldg(cols + m.e0 + lh);
    m.w = __ldg(vals + m.e0 + lh);
  }
  m.b = bias ? __ldg(bias + r) : 0.0f;
}

// stages neighbour rows 0..15 of an item: lane h copies halves (h & 1) of rows h >> 1 and (h >> 1) + 8
__device__ __forceinline__ void issue_rows16(const Row16& m, int64_t word0, bool valid, const uint32_t* state,
                                             int64_t W, unsigned char* buf, int lh) {
  const int staged = valid ? (m.deg < kB16StageRows ? m.deg : kB16StageRows) : 0;
  const int k0 = lh >> 1, half = lh & 1;
  const int32_t j0 = __shfl_sync(kFull, m.col, k0, 16);
  const int32_t j1 = __shfl_sync(kFull, m.col, k0 + 8, 16);
  if (k0 < staged) cp_async_bytes<16>(buf + k0 * kB16Slice + half * 16, state + (int64_t)j0 * W + word0 + half * 4);
  if (k0 + 8 < staged)
    cp_async_bytes<16>(buf + (k0 + 8) * kB16Slice + half * 16, state + (int64_t)j1 * W + word0 + half * 4);
}

// out[j] = in[j] + w, out[j + N] = in[j] - w: one more left-to-right term, its
// sign in bit log2(N) of the entry
template <int N>
__device__ __forceinline__ void expand(const float (&in)[N], float w, float (&out)[2 * N]) {
#pragma unroll
  for (int j = 0; j < N; ++j) {
    out[j] = __fadd_rn(in[j], w);
    out[j + N] = __fadd_rn(in[j], -w);
  }
}

// the 256 left-to-right partial sums of +-w_0..+-w_7 (entry bit k set = -w_k);
// lane h of the half writes the 16 entries h | (j << 4)
__device__ __forceinline__ void build_table16(float* T, float wl, int lh) {
  float w[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) w[k] = __shfl_sync(kFull, wl, k, 16);
  const uint32_t l = (uint32_t)lh;
  float v1[1], v2[2], v4[4], v8[8], v16[16];
  v1[0] = __fadd_rn(flip(w[0], (l & 1u) << 31), flip(w[1], ((l >> 1) & 1u) << 31));
  v1[0] = __fadd_rn(v1[0], flip(w[2], ((l >> 2) & 1u) << 31));
  v1[0] = __fadd_rn(v1[0], flip(w[3], ((l >> 3) & 1u) << 31));
  expand(v1, w[4], v2);
  expand(v2, w[5], v4);
  expand(v4, w[6], v8);
  expand(v8, w[7], v16);
#pragma unroll
  for (int j = 0; j < 16; ++j) T[l | (j << 4)] = v16[j];
}

// acc[v] += w * s_v for the 16 chains of a lane, s_v = -1 where bit v of x is set
__device__ __forceinline__ void accumulate16(float (&acc)[16], uint32_t x, float w) {
  const uint32_t wb = __float_as_uint(w);
#pragma unroll
  for (int v = 0; v < 16; ++v) acc[v] = __fadd_rn(acc[v], __uint_as_float(wb ^ ((x << (31 - v)) & 0x80000000u)));
}

template <bool VARIATES>
__global__ void __launch_bounds__(kB16Threads, TTHRML_BITS16_MIN_BLOCKS) k_spin_bits16(
    const int64_t* __restrict__ row_ptr, const int32_t* __restrict__ cols, const float* __restrict__ vals,
    const float* __restrict__ bias, int64_t row_start, int64_t n_rows, uint32_t* state, int64_t W,
    int64_t chain_offset, const float* __restrict__ variates, int64_t variates_sweeps, uint64_t seed,
    uint32_t sweep_base, const tthrml_run_ctl* __restrict__ ctl, const int32_t* __restrict__ row_order) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31, h = lane >> 4, lh = lane & 15;
  unsigned char* hbuf = smem + (size_t)((threadIdx.x >> 5) * 2 + h) * kB16HalfBytes;
  float* table = reinterpret_cast<float*>(hbuf + 2 * kB16StageBytes);
  const int64_t C = W * 32;
  const int64_t slices = W / 8;
  const int64_t items = n_rows * slices;
  const int64_t n_halves = ((int64_t)gridDim.x * blockDim.x) >> 4;
  const int64_t stride = n_halves;
  int64_t item = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
  const uint32_t sweep = sweep_base + (ctl ? ctl->sweep : 0u);
  const uint64_t sd = ctl ? ctl->seed : seed;
  const PhiloxKeys keys = philox_keys(seed_lo(sd), seed_hi(sd));
  const unsigned char* state_bytes = reinterpret_cast<const unsigned char*>(state);
  // item -> (row, slice): items of one row are consecutive; row_order (if given) lists the block's rows
  // in processing order (rows of equal degree side by side keep a warp's two half-warps in step)
  auto row_of = [&](int64_t it) -> int64_t {
    const int64_t ri = slices == 1 ? it : (int64_t)((uint64_t)it / (uint64_t)slices);
    return row_order && it < items ? (int64_t)__ldg(row_order + ri) : ri;
  };
  auto slice_of = [&](int64_t it) -> int64_t { return slices == 1 ? 0 : (int64_t)((uint64_t)it % (uint64_t)slices); };

  Row16 cur, nxt;
  load_row16(row_of(item), item < items, row_ptr, cols, vals, bias, lh, cur);
  int stage = 0;
  issue_rows16(cur, slice_of(item) * 8, item < items, state, W, hbuf, lh);
  cp_async_commit();
  int64_t next = item + stride;
  load_row16(row_of(next), next < items, row_ptr, cols, vals, bias, lh, nxt);

  while (__any_sync(kFull, item < items)) {
    const bool valid = item < items;
    issue_rows16(nxt, slice_of(next) * 8, next < items, state, W, hbuf + (stage ^ 1) * kB16StageBytes,
                 lh);
    cp_async_commit();
    Row16 after;
    load_row16(row_of(next + stride), next + stride < items, row_ptr, cols, vals, bias, lh, after);

    const int64_t slice = slice_of(item);
    const int64_t c0 = slice * 256 + lh * 16;           // first chain of this lane
    const int64_t byte0 = slice * kB16Slice + lh * 2;   // this lane's two bytes within a row
    const int64_t row = row_start + cur.r;
    uint32_t bits[16];
    if (!VARIATES) {  // independent of the neighbour data: computed while it is in flight
      const int64_t g0 = chain_offset + c0;
#pragma unroll
      for (int v = 0; v < 16; v += 4) {
        const u32x4 rr = philox4x32_10(u32x4{(uint32_t)((g0 + v) >> 2), (uint32_t)row, sweep, kSaltSpin}, keys);
        bits[v] = rr.x;
        bits[v + 1] = rr.y;
        bits[v + 2] = rr.z;
        bits[v + 3] = rr.w;
      }
    }

    const int deg = cur.deg;
    const int staged = deg < kB16StageRows ? deg : kB16StageRows;
    const int t = deg < kTableBits ? deg : kTableBits;
    const unsigned char* sbuf = hbuf + stage * kB16StageBytes + 2 * lh;
    __syncwarp();  // the previous items' lookups are finished before the tables are rewritten
    build_table16(table, cur.w, lh);
    cp_async_wait<1>();
    __syncwarp();  // tables and this item's staged rows are visible to the warp
    uint32_t x[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] = k < t ? (uint32_t)*reinterpret_cast<const uint16_t*>(sbuf + k * kB16Slice) : 0u;
    // bytes 0 (chains 0..7 of the lane) and 1 (chains 8..15) of neighbours 0..3 and 4..7
    const uint32_t p01 = __byte_perm(x[0], x[1], 0x5140u), p23 = __byte_perm(x[2], x[3], 0x5140u);
    const uint32_t p45 = __byte_perm(x[4], x[5], 0x5140u), p67 = __byte_perm(x[6], x[7], 0x5140u);
    uint32_t lo0 = __byte_perm(p01, p23, 0x5410u), lo1 = __byte_perm(p01, p23, 0x7632u);
    uint32_t hi0 = __byte_perm(p45, p67, 0x5410u), hi1 = __byte_perm(p45, p67, 0x7632u);
    transpose8x8(lo0, hi0);  // byte v = sign bits of chain v over neighbours 0..7
    transpose8x8(lo1, hi1);  // byte v = sign bits of chain 8 + v
    float acc[16];
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      acc[v] = table[(lo0 >> (8 * v)) & 0xFFu];
      acc[v + 4] = table[(hi0 >> (8 * v)) & 0xFFu];
      acc[v + 8] = table[(lo1 >> (8 * v)) & 0xFFu];
      acc[v + 12] = table[(hi1 >> (8 * v)) & 0xFFu];
    }
    // neighbours 8..15: staged rows (bounds uniform over the two halves for the shuffles)
    const int staged_max = max(staged, __shfl_xor_sync(kFull, staged, 16));
    for (int k = kTableBits; k < staged_max; ++k) {
      const float w = __shfl_sync(kFull, cur.w, k, 16);
      if (k < staged) accumulate16(acc, *reinterpret_cast<const uint16_t*>(sbuf + k * kB16Slice), w);
    }
    // neighbours 16 and up: columns and weights fetched 16 at a time, bytes read directly
    const int deg_max = max(deg, __shfl_xor_sync(kFull, deg, 16));
    for (int eb = 16; eb < deg_max; eb += 16) {
      const int n = deg - eb;  // this half's terms left (may be <= 0)
      const int32_t my_col = lh < n ? __ldg(cols + cur.e0 + eb + lh) : 0;
      const float my_w = lh < n ? __ldg(vals + cur.e0 + eb + lh) : 0.0f;
      const int chunk = min(16, deg_max - eb);
      for (int k = 0; k < chunk; ++k) {
        const int32_t j = __shfl_sync(kFull, my_col, k, 16);
        const float w = __shfl_sync(kFull, my_w, k, 16);
        if (k < n) accumulate16(acc, *reinterpret_cast<const uint16_t*>(state_bytes + (int64_t)j * W * 4 + byte0), w);
      }
    }

    uint32_t down = 0u;  // bit v set = chain v samples -1
    if (VARIATES) {
      if (valid) {
        const int64_t vs = (int64_t)(sweep % (uint32_t)(variates_sweeps > 0 ? variates_sweeps : 1));
        const float* lrow = variates + (vs * n_rows + cur.r) * C + c0;
#pragma unroll
        for (int v = 0; v < 16; ++v) {
          const float gamma = bias ? __fadd_rn(cur.b, acc[v]) : acc[v];
          down |= (__fmul_rn(2.0f, gamma) > __ldg(lrow + v) ? 0u : 1u) << v;
        }
      }
    } else {
#pragma unroll
      for (int v = 0; v < 16; ++v) {
        const float gamma = bias ? __fadd_rn(cur.b, acc[v]) : acc[v];
        down |= (spin_up_fast(gamma, bits[v]) ? 0u : 1u) << v;
      }
    }
    if (valid) *reinterpret_cast<uint16_t*>(reinterpret_cast<unsigned char*>(state) + row * W * 4 + byte0) = (uint16_t)down;

    __syncwarp();  // every lane is done with this stage before it is refilled
    stage ^= 1;
    cur = nxt;
    nxt = after;
    item = next;
    next += stride;
  }
  cp_async_wait<0>();
}

}  // namespace

template <bool VARIATES>
int launch_bits16(const int64_t* rp, const int32_t* cols, const float* vals, const float* bias, int64_t row_start,
                  int64_t n_rows, uint32_t* state, int64_t W, int64_t chain_offset, const float* variates,
                  int64_t variates_sweeps, uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl,
                  const int32_t* row_order, cudaStream_t s) {
  constexpr int smem = (kB16Threads / 16) * kB16HalfBytes;
  static int per_sm = 0, sms = 0;  // same values from every thread: a benign race
  if (!per_sm) {
    int dev = 0, n = 0, b = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_spin_bits16<VARIATES>, kB16Threads, smem);
    if (e != cudaSuccess) return cuda_status(e, "k_spin_bits16 set-up");
    sms = n;
    per_sm = b > 0 ? b : 1;
  }
  const int64_t items = n_rows * (W / 8);
  const int64_t need = (items + kB16Threads / 16 - 1) / (kB16Threads / 16);
  const int64_t full = (int64_t)sms * per_sm;
  const int grid = (int)(need < full ? (need > 0 ? need : 1) : full);
  k_spin_bits16<VARIATES><<<grid, kB16Threads, smem, s>>>(rp, cols, vals, bias, row_start, n_rows, state, W,
                                                          chain_offset, variates, variates_sweeps, seed, sweep, ctl,
                                                          row_order);
  return launch_status("k_spin_bits16 launch");
}

template int launch_bits16<true>(const int64_t*, const int32_t*, const float*, const float*, int64_t, int64_t,
                                 uint32_t*, int64_t, int64_t, const float*, int64_t, uint64_t, uint32_t,
                                 const tthrml_run_ctl*, const int32_t*, cudaStream_t);
template int launch_bits16<false>(const int64_t*, const int32_t*, const float*, const float*, int64_t, int64_t,
                                  uint32_t*, int64_t, int64_t, const float*, int64_t, uint64_t, uint32_t,
                                  const tthrml_run_ctl*, const int32_t*, cudaStream_t);

}  // namespace tthrml
