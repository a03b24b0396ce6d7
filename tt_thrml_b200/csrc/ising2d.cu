// Single-chain 2-D Ising checkerboard half-sweep on a split-colour int8 lattice.
//
// Layout: colour c of an H x W periodic lattice (W % 32 == 0) is an int8 array
// [rows][W/2] of +-1 spins: site (Y, x) of colour c = (x + Y) % 2 sits at row
// Y, column x/2 -- exactly the executor's block-ordered flat state of a
// lattice program with one chain (block row = linear index / 2).  A strip of
// the lattice is the same array restricted to some rows, with halo rows above
// and below holding the neighbours' rows.
//
// One thread updates 16 consecutive sites of a row (one 16-byte vector): the
// other colour's rows Y-1, Y, Y+1 give the up, left/right and down
// neighbours; site j of row Y (x = 2j + p, p = (Y + c) % 2) has its left and
// right neighbours at other-colour columns j-1+p and j+p.  The four sign bits
// (left, right, up, down: the reference lattice's neighbour order) index a
// 16-entry table built on the host from the program's float32 weights:
//   Philox mode: threshold T with "up" iff m < T, the exact integer form of
//     u < sigmoid(2 * gamma) for the 23-bit draw m, u = (2 m + 1) / 2^24;
//   variates mode: the float32 field gamma, "up" iff 2 * gamma > logit.
// gamma is the left-to-right float32 sum of the bias interaction and the
// pair terms (tt_thrml/compiler.py:303-324), so both modes decide as the
// table-driven kernels do.  Philox draws are split uniforms (common.cuh):
// the top 16 bits of m from counter (chain, flat row / 8, sweep, "LSPI"),
// half (flat row % 2) of word (flat row / 2) % 4 -- eight consecutive sites
// of a row per call -- and the low 7 bits from the per-site refill counter,
// read only when the top bits tie with the threshold's.
//
// Uniform lattices (the threshold depends only on the number of -1
// neighbours) run the bit-sliced kernels below instead: k_ising2d_planes on
// the same int8 rows and k_ising2d_bits on bit-packed rows (32 sites per
// uint32), 32 sites per thread in both, with bit-plane draws.
//
// Observables (optional, for the energy/magnetisation trace): the sum of the
// new spins over the counted rows, and in the colour-1 half-sweep the bond
// sum sum_i s_i (s_left + s_right + s_up + s_down), which counts every bond
// of the lattice once; both exact int64, one atomic per CTA.
#include "common.cuh"

namespace tthrml {
namespace {

constexpr int kIsingThreads = 256;
#ifndef TTHRML_ISING_BITS_QUEUE
#define TTHRML_ISING_BITS_QUEUE 1  // k_ising2d_bits: finish undecided words from a per-warp queue
#endif
constexpr int kBitsQueue = 64;  // queue slots per warp: fewer than 32 wait between drains, plus one word per lane
#ifndef TTHRML_ISING_MIN_BLOCKS
#define TTHRML_ISING_MIN_BLOCKS 3
#endif
#ifndef TTHRML_ISING_PLANES_MIN_BLOCKS
#define TTHRML_ISING_PLANES_MIN_BLOCKS 3
#endif
#ifndef TTHRML_ISING_BITS_WORDS
#define TTHRML_ISING_BITS_WORDS 4  // k_ising2d_bits: most words per thread where rows allow (1, 2 or 4)
#endif
#ifndef TTHRML_ISING_BITS2_MIN_BLOCKS
#define TTHRML_ISING_BITS2_MIN_BLOCKS 2  // k_ising2d_bits with two or four words per thread
#endif

__device__ __forceinline__ uint4 ld16(const int8_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

template <bool VARIATES, bool TRACE>
__global__ void __launch_bounds__(kIsingThreads, TTHRML_ISING_MIN_BLOCKS) k_ising2d(
    int8_t* __restrict__ cc, const int8_t* __restrict__ co, int64_t half_w, FastDiv div_chunks, int64_t rows_local,
    int32_t wrap,
    int64_t row_lo, int64_t row_hi, int64_t global_row0, int64_t height, int32_t colour, int64_t block_row0,
    const uint32_t* __restrict__ thresholds, const float* __restrict__ fields, const float* __restrict__ variates,
    int64_t variates_sweeps, int64_t chain, uint64_t seed, uint32_t sweep_base, const tthrml_run_ctl* __restrict__ ctl,
    int64_t count_lo, int64_t count_hi, unsigned long long* __restrict__ trace, int64_t trace_len,
    tthrml_halo_export ex) {
  __shared__ int32_t TH[16];   // threshold >> 7: compared with the draw's top 16 bits
  __shared__ uint32_t TL[16];  // threshold & 127: compared with the refill bits on a tie
  __shared__ float F[16];
  __shared__ long long red[2];
  if (threadIdx.x < 16) {
    if (VARIATES) {
      F[threadIdx.x] = fields[threadIdx.x];
    } else {
      const uint32_t t = thresholds[threadIdx.x];
      TH[threadIdx.x] = (int32_t)(t >> 7);
      TL[threadIdx.x] = t & 127u;
    }
  }
  if (TRACE && threadIdx.x < 2) red[threadIdx.x] = 0;
  __syncthreads();

  const uint32_t sweep = sweep_base + (ctl ? ctl->sweep : 0u);
  const uint64_t sd = ctl ? ctl->seed : seed;
  const PhiloxKeys keys = philox_keys(seed_lo(sd), seed_hi(sd));
  const uint32_t chunks = div_chunks.d;
  const uint32_t items = (uint32_t)(row_hi - row_lo) * chunks;  // < 2^31, checked by the host
  const int64_t vs = VARIATES ? (int64_t)(sweep % (uint32_t)(variates_sweeps > 0 ? variates_sweeps : 1)) : 0;
  long long mag = 0, bonds = 0;

  for (uint32_t it = blockIdx.x * blockDim.x + threadIdx.x; it < items; it += gridDim.x * blockDim.x) {
    const uint32_t ri = fdiv(it, div_chunks);
    const int64_t i = row_lo + ri;                   // local row
    const int64_t j0 = (int64_t)(it - ri * chunks) << 4;  // first column
    int64_t Y = global_row0 + i;
    if (Y >= height) Y -= height;
    if (Y >= height) Y -= height;
    const int p = (int)((Y + colour) & 1);
    const int64_t iu = i == 0 ? (wrap ? rows_local - 1 : 0) : i - 1;
    const int64_t id = i == rows_local - 1 ? (wrap ? 0 : i) : i + 1;
    const int8_t* rowc = co + i * half_w;
    const uint4 mid = ld16(rowc + j0);
    const uint4 up = ld16(co + iu * half_w + j0);
    const uint4 dn = ld16(co + id * half_w + j0);
    // the byte beyond the 16 on the neighbour side (periodic in x)
    const int64_t je = p ? (j0 + 16 == half_w ? 0 : j0 + 16) : (j0 == 0 ? half_w - 1 : j0 - 1);
    const uint32_t edge = (uint32_t)(uint8_t)__ldg(rowc + je);
    const uint32_t m[6] = {p ? 0u : edge << 24, mid.x, mid.y, mid.z, mid.w, p ? edge : 0u};
    const uint32_t uw[4] = {up.x, up.y, up.z, up.w};
    const uint32_t dw[4] = {dn.x, dn.y, dn.z, dn.w};

    const int64_t flat0 = block_row0 + Y * half_w + j0;  // flat row of the first site (a multiple of 16)
    uint32_t outw[4];
    u32x4 rr{0u, 0u, 0u, 0u};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      // neighbour words of sites 4k..4k+3
      const uint32_t L = p ? m[k + 1] : __byte_perm(m[k], m[k + 1], 0x6543u);
      const uint32_t R = p ? __byte_perm(m[k + 1], m[k + 2], 0x4321u) : m[k + 1];
      const uint32_t idx4 = ((L >> 7) & 0x01010101u) | ((R >> 6) & 0x02020202u) | ((uw[k] >> 5) & 0x04040404u) |
                            ((dw[k] >> 4) & 0x08080808u);
      uint32_t minus = 0u;  // byte v 0xFF: site 4k+v samples -1, 0x00: +1
      if (VARIATES) {
        const float* lrow = variates + vs * (height * half_w) + (flat0 - block_row0) + 4 * k;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float g = F[(idx4 >> (8 * v)) & 0xFu];
          minus |= (__fmul_rn(2.0f, g) > __ldg(lrow + v) ? 0u : 0xFFu) << (8 * v);
        }
      } else {
        const int64_t flat = flat0 + 4 * k;
        if ((k & 1) == 0)
          rr = philox4x32_10(u32x4{(uint32_t)chain, (uint32_t)(flat >> 3), sweep, kSaltLatticeSpin}, keys);
        int32_t a[4];  // threshold top bits - draw top bits: > 0 up, < 0 down, 0 tie
        bool tie = false;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const uint32_t wv = word_of(rr, 2 * (k & 1) + (v >> 1));
          const int32_t h = (int32_t)((v & 1) ? (wv >> 16) : (wv & 0xFFFFu));
          a[v] = TH[(idx4 >> (8 * v)) & 0xFu] - h;
          tie |= a[v] == 0;
        }
        // byte v = the sign of a[v] replicated (0xFF when the site goes down)
        minus = prmt_sign(prmt_sign((uint32_t)a[0], (uint32_t)a[1], 0xFFFBu),
                          prmt_sign((uint32_t)a[2], (uint32_t)a[3], 0xFFFBu), 0x5410u);
        if (tie) {  // rare: decide the tied sites on their refill bits
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            if (a[v] == 0) {
              const uint32_t f =
                  philox4x32_10(u32x4{(uint32_t)chain, (uint32_t)(flat + v), sweep, kSaltLatticeRefill}, keys).x >> 25;
              const bool up = f < TL[(idx4 >> (8 * v)) & 0xFu];
              minus = (minus & ~(0xFFu << (8 * v))) | ((up ? 0u : 0xFFu) << (8 * v));
            }
          }
        }
      }
      outw[k] = minus | 0x01010101u;  // +1 -> 0x01, -1 -> 0xFF per byte
      if (TRACE && i >= count_lo && i < count_hi) {
        const int nm = __popc(minus) >> 3;
        mag += 4 - 2 * nm;
        if (colour == 1) {
          // sum_v s_v * n_v with n_v = 4 - 2 k_v (k_v minus neighbours), s_v = 1 - 2 m_v
          const int ksum = __popc(idx4);
          const int mk = __popc(idx4 & minus);
          bonds += 4 * (4 - 2 * nm) - 2 * ksum + 4 * mk;
        }
      }
    }
    const uint4 outv = make_uint4(outw[0], outw[1], outw[2], outw[3]);
    *reinterpret_cast<uint4*>(cc + i * half_w + j0) = outv;
    if (ex.rows) {  // boundary rows also go straight to the neighbours' mailboxes (peer memory)
      const int64_t slot = (int64_t)(((sweep / ex.sweeps_per_period) + 1u) & 1u) * ex.slot_bytes;
      bool sent = false;
      if (ex.up && i >= ex.up_row0 && i < ex.up_row0 + ex.rows) {
        *reinterpret_cast<uint4*>(ex.up + slot + (i - ex.up_row0) * half_w + j0) = outv;
        sent = true;
      }
      if (ex.down && i >= ex.down_row0 && i < ex.down_row0 + ex.rows) {
        *reinterpret_cast<uint4*>(ex.down + slot + (i - ex.down_row0) * half_w + j0) = outv;
        sent = true;
      }
      if (sent) __threadfence_system();
    }
  }
  if (TRACE) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mag += __shfl_xor_sync(0xffffffffu, mag, o);
      bonds += __shfl_xor_sync(0xffffffffu, bonds, o);
    }
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(&red[0]), (unsigned long long)mag);
      atomicAdd(reinterpret_cast<unsigned long long*>(&red[1]), (unsigned long long)bonds);
    }
    __syncthreads();
    if (threadIdx.x == 0 && (int64_t)sweep < trace_len) {
      atomicAdd(trace + 2 * (int64_t)sweep, (unsigned long long)red[0]);
      if (colour == 1) atomicAdd(trace + 2 * (int64_t)sweep + 1, (unsigned long long)red[1]);
    }
  }
}

// Bit-sliced variant for count-symmetric tables (the threshold depends only on
// the number n of -1 neighbours, as on every uniform lattice), Philox mode.
// A thread updates 32 consecutive sites of a row, held as 32-bit masks in
// byte-transposed order: site s = 4j + k of the chunk is bit 8k + j (byte k of
// int8 word j of the row lands in bit 8k + j with one shift and one masked OR).
// The neighbour masks L, R, U, D (bit set = -1) give the count n in three
// bit-planes (a small adder); the draw m of a site is compared with T(n) one
// bit at a time from the top, for all 32 sites at once: per plane the
// threshold bit T_b(n) is a 5-way select of the plane's per-count masks (0 or
// ~0, in shared memory), and lt |= eq & T_b & ~u_b, eq &= ~(T_b ^ u_b) with u_b
// the draws' bits.  A thread stops once no site is tied, on average after
// three Philox calls for the 32 sites (four planes per call) instead of four
// calls per 16 sites.  Random bits ("planes" layout): plane b (bit 22 - b of
// m) of the 32-site group g = flat row / 32 is word b % 4 of counter (chain,
// g, sweep, "LPL0" + b / 4), site s at bit 8 (s % 4) + s / 4.  The decision is
// exactly m < T(n): with every plane tied, m == T(n) and the site goes down.
template <bool TRACE>
__global__ void __launch_bounds__(kIsingThreads, TTHRML_ISING_PLANES_MIN_BLOCKS) k_ising2d_planes(
    int8_t* __restrict__ cc, const int8_t* __restrict__ co, int64_t half_w, FastDiv div_chunks, int64_t rows_local,
    int32_t wrap, int64_t row_lo, int64_t row_hi, int64_t global_row0, int64_t height, int32_t colour,
    int64_t block_row0, const uint32_t* __restrict__ thresholds, int64_t chain, uint64_t seed, uint32_t sweep_base,
    const tthrml_run_ctl* __restrict__ ctl, int64_t count_lo, int64_t count_hi, unsigned long long* __restrict__ trace,
    int64_t trace_len, tthrml_halo_export ex) {
  // MS[i][n]: bit 23 - i of the count-n threshold as a 0 / ~0 mask (row 0: bit 23, set only for T = 2^23)
  __shared__ __align__(16) uint32_t MS[24][8];
  __shared__ long long red[2];
  planes_masks(MS, thresholds);
  if (TRACE && threadIdx.x < 2) red[threadIdx.x] = 0;
  __syncthreads();

  const uint32_t sweep = sweep_base + (ctl ? ctl->sweep : 0u);
  const uint64_t sd = ctl ? ctl->seed : seed;
  const PhiloxKeys keys = philox_keys(seed_lo(sd), seed_hi(sd));
  const uint32_t chunks = div_chunks.d;
  const uint32_t items = (uint32_t)(row_hi - row_lo) * chunks;  // < 2^31, checked by the host
  long long mag = 0, bonds = 0;

  for (uint32_t it = blockIdx.x * blockDim.x + threadIdx.x; it < items; it += gridDim.x * blockDim.x) {
    const uint32_t ri = fdiv(it, div_chunks);
    const int64_t i = row_lo + ri;
    const int64_t j0 = (int64_t)(it - ri * chunks) << 5;
    int64_t Y = global_row0 + i;
    if (Y >= height) Y -= height;
    if (Y >= height) Y -= height;
    const int p = (int)((Y + colour) & 1);
    const int64_t iu = i == 0 ? (wrap ? rows_local - 1 : 0) : i - 1;
    const int64_t id = i == rows_local - 1 ? (wrap ? 0 : i) : i + 1;
    const int8_t* rowc = co + i * half_w + j0;
    const int8_t* rowu = co + iu * half_w + j0;
    const int8_t* rowd = co + id * half_w + j0;
    const uint4 m0 = ld16(rowc), m1 = ld16(rowc + 16);
    const uint4 u0 = ld16(rowu), u1 = ld16(rowu + 16);
    const uint4 d0 = ld16(rowd), d1 = ld16(rowd + 16);
    const int64_t je = p ? (j0 + 32 == half_w ? 0 : j0 + 32) : (j0 == 0 ? half_w - 1 : j0 - 1);
    const uint32_t e = ((uint32_t)(uint8_t)__ldg(co + i * half_w + je)) >> 7;  // 1: the edge neighbour is -1
    auto signs = [](const uint4& a, const uint4& b) -> uint32_t {
      const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      uint32_t acc = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) acc |= (w[j] >> (7 - j)) & (0x01010101u << j);
      return acc;
    };
    const uint32_t M = signs(m0, m1), U = signs(u0, u1), D = signs(d0, d1);
    // site s - 1 (left, p = 0) and s + 1 (right, p = 1) in byte-transposed order
    const uint32_t L = p ? M : sites_minus1(M, e);
    const uint32_t R = p ? sites_plus1(M, e) : M;
    const uint32_t g32 = (uint32_t)((block_row0 + Y * half_w + j0) >> 5);
    const uint32_t dn = planes_decide(L, R, U, D, MS, (uint32_t)chain, g32, sweep, keys);  // bit set: -1
    uint32_t outw[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) outw[j] = ((dn >> j) & 0x01010101u) * 0xFEu + 0x01010101u;  // +1: 0x01, -1: 0xFF
    if (TRACE && i >= count_lo && i < count_hi) {
      const int nd = __popc(dn);
      mag += 32 - 2 * nd;
      if (colour == 1) {
        const int ksum = __popc(L) + __popc(R) + __popc(U) + __popc(D);
        const int mk = __popc(dn & L) + __popc(dn & R) + __popc(dn & U) + __popc(dn & D);
        bonds += 4 * (32 - 2 * nd) - 2 * ksum + 4 * mk;
      }
    }
    const uint4 o0 = make_uint4(outw[0], outw[1], outw[2], outw[3]);
    const uint4 o1 = make_uint4(outw[4], outw[5], outw[6], outw[7]);
    int8_t* dst = cc + i * half_w + j0;
    *reinterpret_cast<uint4*>(dst) = o0;
    *reinterpret_cast<uint4*>(dst + 16) = o1;
    if (ex.rows) {  // boundary rows also go straight to the neighbours' mailboxes (peer memory)
      const int64_t slot = (int64_t)(((sweep / ex.sweeps_per_period) + 1u) & 1u) * ex.slot_bytes;
      bool sent = false;
      if (ex.up && i >= ex.up_row0 && i < ex.up_row0 + ex.rows) {
        int8_t* q = ex.up + slot + (i - ex.up_row0) * half_w + j0;
        *reinterpret_cast<uint4*>(q) = o0;
        *reinterpret_cast<uint4*>(q + 16) = o1;
        sent = true;
      }
      if (ex.down && i >= ex.down_row0 && i < ex.down_row0 + ex.rows) {
        int8_t* q = ex.down + slot + (i - ex.down_row0) * half_w + j0;
        *reinterpret_cast<uint4*>(q) = o0;
        *reinterpret_cast<uint4*>(q + 16) = o1;
        sent = true;
      }
      if (sent) __threadfence_system();
    }
  }
  if (TRACE) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mag += __shfl_xor_sync(0xffffffffu, mag, o);
      bonds += __shfl_xor_sync(0xffffffffu, bonds, o);
    }
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(&red[0]), (unsigned long long)mag);
      atomicAdd(reinterpret_cast<unsigned long long*>(&red[1]), (unsigned long long)bonds);
    }
    __syncthreads();
    if (threadIdx.x == 0 && (int64_t)sweep < trace_len) {
      atomicAdd(trace + 2 * (int64_t)sweep, (unsigned long long)red[0]);
      if (colour == 1) atomicAdd(trace + 2 * (int64_t)sweep + 1, (unsigned long long)red[1]);
    }
  }
}

// The bit-sliced half-sweep on bit-packed rows: colour c of the strip is a
// uint32 array [rows][W/64], word w of a row holding sites 32w .. 32w + 31 in
// the byte-transposed order of k_ising2d_planes (site s at bit 8 (s % 4) +
// s / 4), bit set = -1.  A thread updates one word: the other colour's words
// at rows i - 1, i, i + 1 are the up, middle and down masks, the left or right
// edge bit comes from the neighbouring word of the middle row, and the
// decision and random bits are those of k_ising2d_planes, so both kernels
// produce the same lattice.  Rows are 8x smaller than int8 rows and need no
// sign gathering; the halo export stores words.  With NW = 4 (rows of a
// multiple of 4 words, 16-byte aligned; else NW = 2 for an even number of
// 8-byte aligned words) a thread takes NW adjacent words of a row: one vector
// load each of the middle, up and down rows and one edge word serve all of
// them, the row arithmetic is shared, and the words' Philox and plane chains
// are independent work for the same warp slot.
template <bool TRACE, int NW>
__global__ void __launch_bounds__(kIsingThreads, NW >= 2 ? TTHRML_ISING_BITS2_MIN_BLOCKS : TTHRML_ISING_PLANES_MIN_BLOCKS)
    k_ising2d_bits(
    uint32_t* __restrict__ cc, const uint32_t* __restrict__ co, int64_t words, FastDiv div_words, int64_t rows_local,
    int32_t wrap, int64_t row_lo, int64_t row_hi, int64_t global_row0, int64_t height, int32_t colour,
    int64_t block_row0, const uint32_t* __restrict__ thresholds, int64_t chain, uint64_t seed, uint32_t sweep_base,
    const tthrml_run_ctl* __restrict__ ctl, int64_t count_lo, int64_t count_hi, unsigned long long* __restrict__ trace,
    int64_t trace_len, tthrml_halo_export ex) {
  __shared__ __align__(16) uint32_t MS[24][8];
  __shared__ long long red[2];
#if TTHRML_ISING_BITS_QUEUE
  __shared__ uint32_t bits_queue[kIsingThreads / 32][7][kBitsQueue];
#endif
  planes_masks(MS, thresholds);
  if (TRACE && threadIdx.x < 2) red[threadIdx.x] = 0;
  __syncthreads();

  const uint32_t sweep = sweep_base + (ctl ? ctl->sweep : 0u);
  const uint64_t sd = ctl ? ctl->seed : seed;
  const PhiloxKeys keys = philox_keys(seed_lo(sd), seed_hi(sd));
  const int64_t half_w = words * 32;
  const uint32_t items = (uint32_t)(row_hi - row_lo) * (uint32_t)words;  // < 2^31, checked by the host
  long long mag = 0, bonds = 0;

#if TTHRML_ISING_BITS_QUEUE
  // Words whose 32 draws are not all decided after the first two Philox chunks (8 bit planes; about 12 %
  // of words) are queued per warp and finished 32 at a time, so the rare third chunk runs with every
  // lane busy instead of stalling whole warps; the planes and their order are those of planes_decide.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t (*q)[kBitsQueue] = bits_queue[warp];  // [L, R, U, D, lt, eq, item][slot]
  int qn = 0;                                    // queued words of this warp (the same in every lane)
  auto locate = [&](uint32_t it, int64_t& i, int64_t& w, int64_t& Y) {
    const uint32_t ri = fdiv(it, div_words);
    i = row_lo + ri;
    w = (int64_t)(it - ri * (uint32_t)words);
    Y = global_row0 + i;
    if (Y >= height) Y -= height;
    if (Y >= height) Y -= height;
  };
  auto finish = [&](uint32_t it, uint32_t L, uint32_t R, uint32_t U, uint32_t D, uint32_t dn) {
    int64_t i, w, Y;
    locate(it, i, w, Y);
    if (TRACE && i >= count_lo && i < count_hi) {
      const int nd = __popc(dn);
      mag += 32 - 2 * nd;
      if (colour == 1) {
        const int ksum = __popc(L) + __popc(R) + __popc(U) + __popc(D);
        const int mk = __popc(dn & L) + __popc(dn & R) + __popc(dn & U) + __popc(dn & D);
        bonds += 4 * (32 - 2 * nd) - 2 * ksum + 4 * mk;
      }
    }
    cc[i * words + w] = dn;
    if (ex.rows) {  // boundary rows also go straight to the neighbours' mailboxes (peer memory)
      const int64_t slot = (int64_t)(((sweep / ex.sweeps_per_period) + 1u) & 1u) * ex.slot_bytes;
      bool sent = false;
      if (ex.up && i >= ex.up_row0 && i < ex.up_row0 + ex.rows) {
        reinterpret_cast<uint32_t*>(ex.up + slot)[(i - ex.up_row0) * words + w] = dn;
        sent = true;
      }
      if (ex.down && i >= ex.down_row0 && i < ex.down_row0 + ex.rows) {
        reinterpret_cast<uint32_t*>(ex.down + slot)[(i - ex.down_row0) * words + w] = dn;
        sent = true;
      }
      if (sent) __threadfence_system();
    }
  };
  auto drain = [&](int first, int n) {  // finish queue slots [first, first + n), one per lane
    __syncwarp();
    if (lane < n) {
      const int k = first + lane;
      const uint32_t L = q[0][k], R = q[1][k], U = q[2][k], D = q[3][k], it = q[6][k];
      PlaneState st;
      plane_counts(st, L, R, U, D);
      st.lt = q[4][k];
      st.eq = q[5][k];
      int64_t i, w, Y;
      locate(it, i, w, Y);
      const uint32_t g32 = (uint32_t)((block_row0 + Y * half_w + 32 * w) >> 5);
#pragma unroll 1
      for (int ch = 2; ch < 6 && st.eq; ++ch)
        planes_chunk(st, MS, philox4x32_10(u32x4{(uint32_t)chain, g32, sweep, kSaltLatticePlanes + (uint32_t)ch}, keys),
                     ch);
      finish(it, L, R, U, D, ~st.lt);
    }
    __syncwarp();
  };
  const uint32_t stride = gridDim.x * blockDim.x;
  const uint32_t groups = items / NW;  // words % NW == 0 (the launcher's choice)
  for (uint32_t g0 = blockIdx.x * blockDim.x + threadIdx.x - lane; g0 < groups; g0 += stride) {
    const uint32_t it = (g0 + lane) * NW;  // this lane's first word
    bool pend[NW];
    uint32_t L[NW], R[NW], U[NW], D[NW];
    PlaneState st[NW];
#pragma unroll
    for (int k = 0; k < NW; ++k) {
      pend[k] = false;
      L[k] = R[k] = U[k] = D[k] = 0u;
      st[k].lt = 0u;
      st[k].eq = 0u;
    }
    if (g0 + lane < groups) {
      int64_t i, w, Y;
      locate(it, i, w, Y);
      const int p = (int)((Y + colour) & 1);
      const int64_t iu = i == 0 ? (wrap ? rows_local - 1 : 0) : i - 1;
      const int64_t id = i == rows_local - 1 ? (wrap ? 0 : i) : i + 1;
      const uint32_t* rowc = co + i * words;
      uint32_t M[NW];
      if constexpr (NW == 4) {
        const uint4 m = __ldg(reinterpret_cast<const uint4*>(rowc + w));
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(co + iu * words + w));
        const uint4 d = __ldg(reinterpret_cast<const uint4*>(co + id * words + w));
        const uint32_t mv[4] = {m.x, m.y, m.z, m.w}, uv[4] = {u.x, u.y, u.z, u.w}, dv[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
        for (int k = 0; k < NW; ++k) {
          M[k] = mv[k];
          U[k] = uv[k];
          D[k] = dv[k];
        }
      } else if constexpr (NW == 2) {
        const uint2 m = __ldg(reinterpret_cast<const uint2*>(rowc + w));
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(co + iu * words + w));
        const uint2 d = __ldg(reinterpret_cast<const uint2*>(co + id * words + w));
        M[0] = m.x;
        M[1] = m.y;
        U[0] = u.x;
        U[1] = u.y;
        D[0] = d.x;
        D[1] = d.y;
      } else {
        M[0] = __ldg(rowc + w);
        U[0] = __ldg(co + iu * words + w);
        D[0] = __ldg(co + id * words + w);
      }
      if (p) {  // right neighbours: site 0 of the next word (bit 0) is the edge
        const uint32_t edge = __ldg(rowc + (w + NW == words ? 0 : w + NW));
#pragma unroll
        for (int k = 0; k < NW; ++k) {
          L[k] = M[k];
          R[k] = sites_plus1(M[k], (k + 1 < NW ? M[(k + 1) % NW] : edge) & 1u);
        }
      } else {  // left neighbours: site 31 of the previous word (bit 31) is the edge
        const uint32_t edge = __ldg(rowc + (w == 0 ? words - 1 : w - 1));
#pragma unroll
        for (int k = 0; k < NW; ++k) {
          L[k] = sites_minus1(M[k], (k > 0 ? M[(k + NW - 1) % NW] : edge) >> 31);
          R[k] = M[k];
        }
      }
      // word w + k draws from counter g32 + k: (x + 32k) >> 5 = (x >> 5) + k
      const uint32_t g32 = (uint32_t)((block_row0 + Y * half_w + 32 * w) >> 5);
#pragma unroll
      for (int k = 0; k < NW; ++k) planes_begin(st[k], L[k], R[k], U[k], D[k], MS);
#pragma unroll
      for (int ch = 0; ch < 2; ++ch)
#pragma unroll
        for (int k = 0; k < NW; ++k)
          planes_chunk(st[k], MS,
                       philox4x32_10(u32x4{(uint32_t)chain, g32 + (uint32_t)k, sweep, kSaltLatticePlanes + (uint32_t)ch},
                                     keys),
                       ch);
#pragma unroll
      for (int k = 0; k < NW; ++k) {
        pend[k] = st[k].eq != 0u;
        if (!pend[k]) finish(it + k, L[k], R[k], U[k], D[k], ~st[k].lt);  // bit set: -1
      }
    }
#pragma unroll
    for (int k = 0; k < NW; ++k) {
      const uint32_t pm = __ballot_sync(0xffffffffu, pend[k]);
      if (pm) {
        if (pend[k]) {
          const int slot = qn + __popc(pm & ((1u << lane) - 1u));
          q[0][slot] = L[k];
          q[1][slot] = R[k];
          q[2][slot] = U[k];
          q[3][slot] = D[k];
          q[4][slot] = st[k].lt;
          q[5][slot] = st[k].eq;
          q[6][slot] = it + k;
        }
        qn += __popc(pm);
        if (qn >= 32) {
          drain(qn - 32, 32);
          qn -= 32;
        }
      }
    }
  }
  if (qn > 0) drain(0, qn);
#else
  static_assert(NW == 1, "two words per thread need the queued loop");
  for (uint32_t it = blockIdx.x * blockDim.x + threadIdx.x; it < items; it += gridDim.x * blockDim.x) {
    const uint32_t ri = fdiv(it, div_words);
    const int64_t i = row_lo + ri;
    const int64_t w = (int64_t)(it - ri * (uint32_t)words);
    int64_t Y = global_row0 + i;
    if (Y >= height) Y -= height;
    if (Y >= height) Y -= height;
    const int p = (int)((Y + colour) & 1);
    const int64_t iu = i == 0 ? (wrap ? rows_local - 1 : 0) : i - 1;
    const int64_t id = i == rows_local - 1 ? (wrap ? 0 : i) : i + 1;
    const uint32_t* rowc = co + i * words;
    const uint32_t M = __ldg(rowc + w);
    const uint32_t U = __ldg(co + iu * words + w), D = __ldg(co + id * words + w);
    uint32_t L, R;
    if (p) {  // right neighbours: site 0 of the next word (bit 0) is the edge
      L = M;
      R = sites_plus1(M, __ldg(rowc + (w + 1 == words ? 0 : w + 1)) & 1u);
    } else {  // left neighbours: site 31 of the previous word (bit 31) is the edge
      L = sites_minus1(M, __ldg(rowc + (w == 0 ? words - 1 : w - 1)) >> 31);
      R = M;
    }
    const uint32_t g32 = (uint32_t)((block_row0 + Y * half_w + 32 * w) >> 5);
    const uint32_t dn = planes_decide(L, R, U, D, MS, (uint32_t)chain, g32, sweep, keys);  // bit set: -1
    if (TRACE && i >= count_lo && i < count_hi) {
      const int nd = __popc(dn);
      mag += 32 - 2 * nd;
      if (colour == 1) {
        const int ksum = __popc(L) + __popc(R) + __popc(U) + __popc(D);
        const int mk = __popc(dn & L) + __popc(dn & R) + __popc(dn & U) + __popc(dn & D);
        bonds += 4 * (32 - 2 * nd) - 2 * ksum + 4 * mk;
      }
    }
    cc[i * words + w] = dn;
    if (ex.rows) {  // boundary rows also go straight to the neighbours' mailboxes (peer memory)
      const int64_t slot = (int64_t)(((sweep / ex.sweeps_per_period) + 1u) & 1u) * ex.slot_bytes;
      bool sent = false;
      if (ex.up && i >= ex.up_row0 && i < ex.up_row0 + ex.rows) {
        reinterpret_cast<uint32_t*>(ex.up + slot)[(i - ex.up_row0) * words + w] = dn;
        sent = true;
      }
      if (ex.down && i >= ex.down_row0 && i < ex.down_row0 + ex.rows) {
        reinterpret_cast<uint32_t*>(ex.down + slot)[(i - ex.down_row0) * words + w] = dn;
        sent = true;
      }
      if (sent) __threadfence_system();
    }
  }
#endif
  if (TRACE) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mag += __shfl_xor_sync(0xffffffffu, mag, o);
      bonds += __shfl_xor_sync(0xffffffffu, bonds, o);
    }
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(&red[0]), (unsigned long long)mag);
      atomicAdd(reinterpret_cast<unsigned long long*>(&red[1]), (unsigned long long)bonds);
    }
    __syncthreads();
    if (threadIdx.x == 0 && (int64_t)sweep < trace_len) {
      atomicAdd(trace + 2 * (int64_t)sweep, (unsigned long long)red[0]);
      if (colour == 1) atomicAdd(trace + 2 * (int64_t)sweep + 1, (unsigned long long)red[1]);
    }
  }
}

template <bool TRACE, int NW>
int launch_ising_bits_nw(uint32_t* cc, const uint32_t* co, int64_t words, int64_t rows_local, int32_t wrap,
                         int64_t row_lo, int64_t row_hi, int64_t global_row0, int64_t height, int32_t colour,
                         int64_t block_row0, const uint32_t* thresholds, int64_t chain, uint64_t seed, uint32_t sweep,
                         const tthrml_run_ctl* ctl, int64_t count_lo, int64_t count_hi, unsigned long long* trace,
                         int64_t trace_len, const tthrml_halo_export& ex, cudaStream_t s) {
  static int per_sm = 0, sms = 0;  // same values from every thread: a benign race
  if (!per_sm) {
    int dev = 0, n = 0, b = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_ising2d_bits<TRACE, NW>, kIsingThreads, 0);
    if (e != cudaSuccess) return cuda_status(e, "k_ising2d_bits set-up");
    sms = n;
    per_sm = b > 0 ? b : 1;
  }
  const int64_t groups = (row_hi - row_lo) * words / NW;
  const int64_t need = (groups + kIsingThreads - 1) / kIsingThreads;
  const int64_t full = (int64_t)sms * per_sm;
  const int grid = (int)(need < full ? (need > 0 ? need : 1) : full);
  k_ising2d_bits<TRACE, NW><<<grid, kIsingThreads, 0, s>>>(
      cc, co, words, make_fastdiv((uint32_t)words), rows_local, wrap, row_lo, row_hi, global_row0, height, colour,
      block_row0, thresholds, chain, seed, sweep, ctl, count_lo, count_hi, trace, trace_len, ex);
  return launch_status("k_ising2d_bits launch");
}

// four (or two) words per thread where the rows' word count and alignment allow
template <bool TRACE>
int launch_ising_bits(uint32_t* cc, const uint32_t* co, int64_t words, int64_t rows_local, int32_t wrap,
                      int64_t row_lo, int64_t row_hi, int64_t global_row0, int64_t height, int32_t colour,
                      int64_t block_row0, const uint32_t* thresholds, int64_t chain, uint64_t seed, uint32_t sweep,
                      const tthrml_run_ctl* ctl, int64_t count_lo, int64_t count_hi, unsigned long long* trace,
                      int64_t trace_len, const tthrml_halo_export& ex, cudaStream_t s) {
#if TTHRML_ISING_BITS_QUEUE && TTHRML_ISING_BITS_WORDS == 4
  if (words % 4 == 0 && reinterpret_cast<uintptr_t>(co) % 16 == 0)
    return launch_ising_bits_nw<TRACE, 4>(cc, co, words, rows_local, wrap, row_lo, row_hi, global_row0, height, colour,
                                          block_row0, thresholds, chain, seed, sweep, ctl, count_lo, count_hi, trace,
                                          trace_len, ex, s);
#endif
#if TTHRML_ISING_BITS_QUEUE && TTHRML_ISING_BITS_WORDS >= 2
  if (words % 2 == 0 && reinterpret_cast<uintptr_t>(co) % 8 == 0)
    return launch_ising_bits_nw<TRACE, 2>(cc, co, words, rows_local, wrap, row_lo, row_hi, global_row0, height, colour,
                                          block_row0, thresholds, chain, seed, sweep, ctl, count_lo, count_hi, trace,
                                          trace_len, ex, s);
#endif
  return launch_ising_bits_nw<TRACE, 1>(cc, co, words, rows_local, wrap, row_lo, row_hi, global_row0, height, colour,
                                        block_row0, thresholds, chain, seed, sweep, ctl, count_lo, count_hi, trace,
                                        trace_len, ex, s);
}

template <bool TRACE>
int launch_ising_planes(int8_t* cc, const int8_t* co, int64_t half_w, int64_t rows_local, int32_t wrap,
                        int64_t row_lo, int64_t row_hi, int64_t global_row0, int64_t height, int32_t colour,
                        int64_t block_row0, const uint32_t* thresholds, int64_t chain, uint64_t seed, uint32_t sweep,
                        const tthrml_run_ctl* ctl, int64_t count_lo, int64_t count_hi, unsigned long long* trace,
                        int64_t trace_len, const tthrml_halo_export& ex, cudaStream_t s) {
  static int per_sm = 0, sms = 0;  // same values from every thread: a benign race
  if (!per_sm) {
    int dev = 0, n = 0, b = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_ising2d_planes<TRACE>, kIsingThreads, 0);
    if (e != cudaSuccess) return cuda_status(e, "k_ising2d_planes set-up");
    sms = n;
    per_sm = b > 0 ? b : 1;
  }
  const int64_t items = (row_hi - row_lo) * (half_w >> 5);
  const int64_t need = (items + kIsingThreads - 1) / kIsingThreads;
  const int64_t full = (int64_t)sms * per_sm;
  const int grid = (int)(need < full ? (need > 0 ? need : 1) : full);
  k_ising2d_planes<TRACE><<<grid, kIsingThreads, 0, s>>>(
      cc, co, half_w, make_fastdiv((uint32_t)(half_w >> 5)), rows_local, wrap, row_lo, row_hi, global_row0, height,
      colour, block_row0, thresholds, chain, seed, sweep, ctl, count_lo, count_hi, trace, trace_len, ex);
  return launch_status("k_ising2d_planes launch");
}

template <bool VARIATES, bool TRACE>
int launch_ising(int8_t* cc, const int8_t* co, int64_t half_w, int64_t rows_local, int32_t wrap, int64_t row_lo,
                 int64_t row_hi, int64_t global_row0, int64_t height, int32_t colour, int64_t block_row0,
                 const uint32_t* thresholds, const float* fields, const float* variates, int64_t variates_sweeps,
                 int64_t chain, uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl, int64_t count_lo,
                 int64_t count_hi, unsigned long long* trace, int64_t trace_len, const tthrml_halo_export& ex,
                 cudaStream_t s) {
  static int per_sm = 0, sms = 0;  // same values from every thread: a benign race
  if (!per_sm) {
    int dev = 0, n = 0, b = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_ising2d<VARIATES, TRACE>, kIsingThreads, 0);
    if (e != cudaSuccess) return cuda_status(e, "k_ising2d set-up");
    sms = n;
    per_sm = b > 0 ? b : 1;
  }
  const int64_t items = (row_hi - row_lo) * (half_w >> 4);
  const int64_t need = (items + kIsingThreads - 1) / kIsingThreads;
  const int64_t full = (int64_t)sms * per_sm;
  const int grid = (int)(need < full ? (need > 0 ? need : 1) : full);
  k_ising2d<VARIATES, TRACE><<<grid, kIsingThreads, 0, s>>>(
      cc, co, half_w, make_fastdiv((uint32_t)(half_w >> 4)), rows_local, wrap, row_lo, row_hi, global_row0, height, colour, block_row0, thresholds, fields,
      variates, variates_sweeps, chain, seed, sweep, ctl, count_lo, count_hi, trace, trace_len, ex);
  return launch_status("k_ising2d launch");
}

}  // namespace
}  // namespace tthrml

namespace {
int halfsweep_impl(int8_t* colour_state, const int8_t* other_state, int64_t width, int64_t rows_local,
                   int32_t wrap_rows, int64_t row_lo, int64_t row_hi, int64_t global_row0, int64_t height,
                   int32_t colour, int64_t block_row0, const uint32_t* thresholds, const float* fields,
                   const float* variates, int64_t variates_sweeps, int64_t chain, uint64_t seed, uint32_t sweep,
                   const tthrml_run_ctl* ctl, int64_t count_lo, int64_t count_hi, int64_t* trace, int64_t trace_len,
                   const tthrml_halo_export* export_host, void* stream, bool planes) {
  using namespace tthrml;
  tthrml_halo_export ex{};
  if (export_host) {
    ex = *export_host;
    if (ex.rows < 0 || (ex.rows && (ex.sweeps_per_period == 0 || ex.slot_bytes < ex.rows * (width / 2) ||
                                    ((uintptr_t)ex.up % 16) || ((uintptr_t)ex.down % 16) || ex.up_row0 < 0 ||
                                    ex.down_row0 < 0 || ex.up_row0 + ex.rows > rows_local ||
                                    ex.down_row0 + ex.rows > rows_local))) {
      set_error("tthrml_ising2d_halfsweep_x: invalid halo export descriptor");
      return TTHRML_ERR_ARG;
    }
  }
  if (!colour_state || !other_state || (colour != 0 && colour != 1)) {
    set_error("tthrml_ising2d_halfsweep: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  if (width <= 0 || width % 32 || height <= 0 || height % 2 || rows_local <= 0) {
    set_error("tthrml_ising2d_halfsweep: width must be a positive multiple of 32 and height positive and even "
              "(got %lld x %lld)", (long long)height, (long long)width);
    return TTHRML_ERR_ARG;
  }
  if (row_lo < 0 || row_hi > rows_local || row_lo > row_hi || global_row0 < 0 || global_row0 >= height ||
      rows_local > 2 * height) {
    set_error("tthrml_ising2d_halfsweep: row range [%lld, %lld) outside the %lld local rows", (long long)row_lo,
              (long long)row_hi, (long long)rows_local);
    return TTHRML_ERR_ARG;
  }
  if (!wrap_rows && (row_lo < 1 || row_hi > rows_local - 1)) {
    set_error("tthrml_ising2d_halfsweep: without wrapping, updated rows need a halo row on both sides");
    return TTHRML_ERR_ARG;
  }
  if (wrap_rows && rows_local != height) {
    set_error("tthrml_ising2d_halfsweep: wrapping rows needs the whole lattice (rows_local == height)");
    return TTHRML_ERR_ARG;
  }
  if (variates ? !fields : !thresholds) {
    set_error("tthrml_ising2d_halfsweep: %s table missing", variates ? "field" : "threshold");
    return TTHRML_ERR_ARG;
  }
  if (((uintptr_t)colour_state % 16) || ((uintptr_t)other_state % 16) || (variates && (uintptr_t)variates % 16)) {
    set_error("tthrml_ising2d_halfsweep: buffers must be 16-byte aligned");
    return TTHRML_ERR_ARG;
  }
  if ((row_hi - row_lo) * (width / 32) >= (1ll << 31)) {
    set_error("tthrml_ising2d_halfsweep: more than 2^31 16-site chunks in one launch");
    return TTHRML_ERR_UNSUPPORTED;
  }
  if (planes && (variates || width % 64 || block_row0 % 32)) {
    set_error("tthrml_ising2d_halfsweep_planes: Philox mode only, width %% 64 == 0 and block_row0 %% 32 == 0 "
              "(got width %lld, block_row0 %lld)", (long long)width, (long long)block_row0);
    return TTHRML_ERR_ARG;
  }
  if (row_hi == row_lo) return TTHRML_OK;
  cudaStream_t s = (cudaStream_t)stream;
  unsigned long long* tr = reinterpret_cast<unsigned long long*>(trace);
  const int64_t hw = width / 2;
  if (planes) {
    if (trace)
      return launch_ising_planes<true>(colour_state, other_state, hw, rows_local, wrap_rows, row_lo, row_hi,
                                       global_row0, height, colour, block_row0, thresholds, chain, seed, sweep, ctl,
                                       count_lo, count_hi, tr, trace_len, ex, s);
    return launch_ising_planes<false>(colour_state, other_state, hw, rows_local, wrap_rows, row_lo, row_hi,
                                      global_row0, height, colour, block_row0, thresholds, chain, seed, sweep, ctl,
                                      count_lo, count_hi, tr, trace_len, ex, s);
  }
#define TTHRML_ISING_LAUNCH(V, TR)                                                                                  \
  return launch_ising<V, TR>(colour_state, other_state, hw, rows_local, wrap_rows, row_lo, row_hi, global_row0,   \
                             height, colour, block_row0, thresholds, fields, variates, variates_sweeps, chain, seed, \
                             sweep, ctl, count_lo, count_hi, tr, trace_len, ex, s)
  if (variates) {
    if (trace) TTHRML_ISING_LAUNCH(true, true);
    TTHRML_ISING_LAUNCH(true, false);
  }
  if (trace) TTHRML_ISING_LAUNCH(false, true);
  TTHRML_ISING_LAUNCH(false, false);
#undef TTHRML_ISING_LAUNCH
}
}  // namespace

extern "C" int tthrml_ising2d_halfsweep_x(int8_t* colour_state, const int8_t* other_state, int64_t width,
                                          int64_t rows_local, int32_t wrap_rows, int64_t row_lo, int64_t row_hi,
                                          int64_t global_row0, int64_t height, int32_t colour, int64_t block_row0,
                                          const uint32_t* thresholds, const float* fields, const float* variates,
                                          int64_t variates_sweeps, int64_t chain, uint64_t seed, uint32_t sweep,
                                          const tthrml_run_ctl* ctl, int64_t count_lo, int64_t count_hi,
                                          int64_t* trace, int64_t trace_len, const tthrml_halo_export* export_host,
                                          void* stream) {
  return halfsweep_impl(colour_state, other_state, width, rows_local, wrap_rows, row_lo, row_hi, global_row0, height,
                        colour, block_row0, thresholds, fields, variates, variates_sweeps, chain, seed, sweep, ctl,
                        count_lo, count_hi, trace, trace_len, export_host, stream, false);
}

extern "C" int tthrml_ising2d_halfsweep_planes(int8_t* colour_state, const int8_t* other_state, int64_t width,
                                               int64_t rows_local, int32_t wrap_rows, int64_t row_lo, int64_t row_hi,
                                               int64_t global_row0, int64_t height, int32_t colour,
                                               int64_t block_row0, const uint32_t* thresholds, int64_t chain,
                                               uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl,
                                               int64_t count_lo, int64_t count_hi, int64_t* trace, int64_t trace_len,
                                               const tthrml_halo_export* export_host, void* stream) {
  return halfsweep_impl(colour_state, other_state, width, rows_local, wrap_rows, row_lo, row_hi, global_row0, height,
                        colour, block_row0, thresholds, nullptr, nullptr, 0, chain, seed, sweep, ctl, count_lo,
                        count_hi, trace, trace_len, export_host, stream, true);
}

extern "C" int tthrml_ising2d_halfsweep(int8_t* colour_state, const int8_t* other_state, int64_t width,
                                        int64_t rows_local, int32_t wrap_rows, int64_t row_lo, int64_t row_hi,
                                        int64_t global_row0, int64_t height, int32_t colour, int64_t block_row0,
                                        const uint32_t* thresholds, const float* fields, const float* variates,
                                        int64_t variates_sweeps, int64_t chain, uint64_t seed, uint32_t sweep,
                                        const tthrml_run_ctl* ctl, int64_t count_lo, int64_t count_hi,
                                        int64_t* trace, int64_t trace_len, void* stream) {
  return tthrml_ising2d_halfsweep_x(colour_state, other_state, width, rows_local, wrap_rows, row_lo, row_hi,
                                    global_row0, height, colour, block_row0, thresholds, fields, variates,
                                    variates_sweeps, chain, seed, sweep, ctl, count_lo, count_hi, trace, trace_len,
                                    nullptr, stream);
}

extern "C" int tthrml_ising2d_halfsweep_bits(uint32_t* colour_state, const uint32_t* other_state, int64_t width,
                                             int64_t rows_local, int32_t wrap_rows, int64_t row_lo, int64_t row_hi,
                                             int64_t global_row0, int64_t height, int32_t colour, int64_t block_row0,
                                             const uint32_t* thresholds, int64_t chain, uint64_t seed, uint32_t sweep,
                                             const tthrml_run_ctl* ctl, int64_t count_lo, int64_t count_hi,
                                             int64_t* trace, int64_t trace_len,
                                             const tthrml_halo_export* export_host, void* stream) {
  using namespace tthrml;
  const int64_t words = width / 64;
  tthrml_halo_export ex{};
  if (export_host) {
    ex = *export_host;
    if (ex.rows < 0 || (ex.rows && (ex.sweeps_per_period == 0 || ex.slot_bytes < ex.rows * words * 4 ||
                                    ((uintptr_t)ex.up % 4) || ((uintptr_t)ex.down % 4) || ex.slot_bytes % 4 ||
                                    ex.up_row0 < 0 || ex.down_row0 < 0 || ex.up_row0 + ex.rows > rows_local ||
                                    ex.down_row0 + ex.rows > rows_local))) {
      set_error("tthrml_ising2d_halfsweep_bits: invalid halo export descriptor");
      return TTHRML_ERR_ARG;
    }
  }
  if (!colour_state || !other_state || !thresholds || (colour != 0 && colour != 1)) {
    set_error("tthrml_ising2d_halfsweep_bits: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  if (width <= 0 || width % 64 || height <= 0 || height % 2 || rows_local <= 0 || block_row0 % 32) {
    set_error("tthrml_ising2d_halfsweep_bits: width must be a positive multiple of 64, height positive and even, "
              "block_row0 a multiple of 32 (got %lld x %lld, %lld)", (long long)height, (long long)width,
              (long long)block_row0);
    return TTHRML_ERR_ARG;
  }
  if (row_lo < 0 || row_hi > rows_local || row_lo > row_hi || global_row0 < 0 || global_row0 >= height ||
      rows_local > 2 * height) {
    set_error("tthrml_ising2d_halfsweep_bits: row range [%lld, %lld) outside the %lld local rows",
              (long long)row_lo, (long long)row_hi, (long long)rows_local);
    return TTHRML_ERR_ARG;
  }
  if (!wrap_rows && (row_lo < 1 || row_hi > rows_local - 1)) {
    set_error("tthrml_ising2d_halfsweep_bits: without wrapping, updated rows need a halo row on both sides");
    return TTHRML_ERR_ARG;
  }
  if (wrap_rows && rows_local != height) {
    set_error("tthrml_ising2d_halfsweep_bits: wrapping rows needs the whole lattice (rows_local == height)");
    return TTHRML_ERR_ARG;
  }
  if (((uintptr_t)colour_state % 4) || ((uintptr_t)other_state % 4)) {
    set_error("tthrml_ising2d_halfsweep_bits: buffers must be 4-byte aligned");
    return TTHRML_ERR_ARG;
  }
  if ((row_hi - row_lo) * words >= (1ll << 31)) {
    set_error("tthrml_ising2d_halfsweep_bits: more than 2^31 words in one launch");
    return TTHRML_ERR_UNSUPPORTED;
  }
  if (row_hi == row_lo) return TTHRML_OK;
  cudaStream_t s = (cudaStream_t)stream;
  unsigned long long* tr = reinterpret_cast<unsigned long long*>(trace);
  if (trace)
    return launch_ising_bits<true>(colour_state, other_state, words, rows_local, wrap_rows, row_lo, row_hi,
                                   global_row0, height, colour, block_row0, thresholds, chain, seed, sweep, ctl,
                                   count_lo, count_hi, tr, trace_len, ex, s);
  return launch_ising_bits<false>(colour_state, other_state, words, rows_local, wrap_rows, row_lo, row_hi,
                                  global_row0, height, colour, block_row0, thresholds, chain, seed, sweep, ctl,
                                  count_lo, count_hi, tr, trace_len, ex, s);
}
