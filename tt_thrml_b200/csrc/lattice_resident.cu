// Persistent multi-sweep kernel for small 2-D Ising lattices with many chains
// (uniform couplings, periodic): every CTA keeps the whole lattice of its 8
// chains in shared memory and runs any number of checkerboard half-sweeps, with
// the per-chain magnetisation of scheduled samples reduced in the kernel, so a
// whole sampling schedule is one launch.
//
// State: the executor's bit-packed layout, uint32 [rows][C/32] with bit c of a
// row set when chain c is -1; rows are block-ordered (colour c's sites of row
// Y, x at block row Y*W/2 + x/2, see csrc/ising2d.cu).  CTA g owns chains
// 8g..8g+7, i.e. byte g % 4 of word g / 4 of every row, and keeps it as one
// byte per site in shared memory, [2 colours][H][W/2] bytes.
//
// Decision (count-symmetric tables, the uniform lattice): bit-sliced over 4
// sites x 8 chains per 32-bit word with bit-plane draws (PLANES below).
// Otherwise: the four neighbour bytes (left, right, up, down) of a site form
// a word N whose bit 8k + v is neighbour k of chain v; a bit-matrix transpose
// of N (the 8x8 transpose of Warren, "Hacker's Delight" 7-3, with the upper
// four rows zero) turns it into one 4-bit sign pattern per chain, which decides
// against the exact integer threshold of the pattern's float32 field (as in
// csrc/ising2d.cu).  Philox draws are split uniforms (common.cuh): the top 16
// bits of chain c's draw come from counter (c / 8, flat row, sweep, "LSPI"),
// half c % 2 of word (c / 2) % 4 -- one call for the CTA's 8 chains of a site
// -- and the low 7 bits from the refill counter, read only on a tie.
#include "common.cuh"

namespace tthrml {
namespace {

constexpr int kResThreads = 512;
constexpr uint32_t kResWaitLimit = 1u << 20;  // try_wait polls of the half-sweep barrier before giving up
constexpr int32_t kErrHalfSweepWait = 5;       // error code: the half-sweep barrier never completed

__device__ __forceinline__ uint32_t res_smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Bounded wait for the completion of the phase of `bar` with the given parity.
__device__ __forceinline__ bool res_bar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = res_smem_u32(bar);
  for (uint32_t i = 0; i < kResWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ int wrapi(int i, int n) { return i < 0 ? i + n : (i >= n ? i - n : i); }

// PLANES: the bit-sliced decision for count-symmetric tables -- a 32-bit
// shared-memory word is 4 sites x 8 chains (byte k = site j + k, bit v = chain
// v); its neighbour words L, R (byte funnel shifts of the other colour's row),
// U and D give each of the 32 spins its count n of -1 neighbours in three
// bit-planes, and the draws are compared with the count-n thresholds one bit
// at a time from the top (as in csrc/ising2d.cu's k_ising2d_planes).  Random
// bits ("planes8"): bit 22 - b of the draw of chain c at flat row f is bit
// 8 (f % 4) + c % 8 of word b % 4 of counter (c / 8, f / 4, sweep, "LPL0" +
// b / 4).
template <bool PLANES>
__global__ void __launch_bounds__(kResThreads) k_ising2d_resident(
    uint32_t* state, int64_t C, int32_t H, int32_t W, int64_t row0_c0, int64_t row0_c1,
    const uint32_t* __restrict__ thresholds, uint64_t seed, uint32_t sweep0, int32_t colour0, int64_t n_half,
    double* __restrict__ obs, int64_t obs_first, int64_t obs_every, int64_t n_obs, int32_t obs_colours,
    int64_t chain_offset, const tthrml_run_ctl* __restrict__ ctl, int32_t* __restrict__ error, FastDiv div_hw) {
  extern __shared__ __align__(16) unsigned char lat[];  // [2][H][W/2]
  __shared__ int32_t TH[16];   // threshold >> 7: compared with a draw's top 16 bits
  __shared__ uint32_t TL[16];  // threshold & 127: compared with the refill bits on a tie
  // PLANES: MS[i][n] = bit 23 - i of the count-n threshold as a 0 / ~0 mask
  __shared__ __align__(16) uint32_t MS[PLANES ? 24 : 1][8];
  __shared__ int counts[8];
  __shared__ uint64_t half_bar;  // split-phase barrier between half-sweeps, one phase per half-sweep
  const int hw = W >> 1;
  const int half_sites = H * hw;
  const int g = blockIdx.x;  // chain group
  const int64_t words = C >> 5;
  const int word = g >> 2, byte_in_word = g & 3;
  if (threadIdx.x < 16) {
    TH[threadIdx.x] = (int32_t)(thresholds[threadIdx.x] >> 7);
    TL[threadIdx.x] = thresholds[threadIdx.x] & 127u;
  }
  if (PLANES) planes_masks(MS, thresholds);
  if (threadIdx.x == 0)
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(res_smem_u32(&half_bar)), "r"((uint32_t)blockDim.x)
                 : "memory");
  for (int i = threadIdx.x; i < 2 * half_sites; i += blockDim.x) {
    const int c = i / half_sites, r = i - c * half_sites;
    const int64_t row = (c ? row0_c1 : row0_c0) + r;
    lat[i] = (unsigned char)(state[row * words + word] >> (8 * byte_in_word));
  }
  __syncthreads();
  const uint64_t sd = ctl ? ctl->seed : seed;
  const PhiloxKeys keys = philox_keys(seed_lo(sd), seed_hi(sd));
  sweep0 += ctl ? ctl->sweep : 0u;
  const uint32_t gc0 = (uint32_t)(chain_offset + 8 * g);  // global index of the group's first chain

  // Eager Philox words of this thread's first word of a half-sweep: they depend on the counter only, so
  // the words of half-sweep t + 1 are drawn between arriving at and waiting on half-sweep t's barrier.
  auto eager_for = [&](int64_t tt, u32x4 (&pre)[TTHRML_PLANES_EAGER]) {
    const int cc = (int)((colour0 + tt) & 1);
    const int64_t r0 = cc ? row0_c1 : row0_c0;
    planes_eager(pre, gc0 >> 3, (uint32_t)((r0 + 4 * (int64_t)threadIdx.x) >> 2),
                 sweep0 + (uint32_t)((colour0 + tt) >> 1), keys);
  };
  u32x4 pre[TTHRML_PLANES_EAGER];
  if (PLANES && n_half > 0) eager_for(0, pre);
  bool failed = false;
  int64_t next_obs = obs ? obs_first : -1, taken = 0;
  for (int64_t t = 0; t < n_half; ++t) {
    const int c = (int)((colour0 + t) & 1);
    const uint32_t sweep = sweep0 + (uint32_t)((colour0 + t) >> 1);
    unsigned char* mine = lat + c * half_sites;
    const unsigned char* other = lat + (1 - c) * half_sites;
    const int64_t row0 = c ? row0_c1 : row0_c0;
    if (PLANES) {
      const uint32_t* ow = reinterpret_cast<const uint32_t*>(other);
      uint32_t* mw = reinterpret_cast<uint32_t*>(mine);
      const int qw = hw >> 2;  // words per colour row
      for (int q = threadIdx.x; q < (half_sites >> 2); q += blockDim.x) {
        const int r = q << 2;
        const int Y = (int)fdiv((uint32_t)r, div_hw), j = r - Y * hw;
        const int p = (Y + c) & 1;
        const int yu = wrapi(Y - 1, H), yd = wrapi(Y + 1, H);
        const int wq = j >> 2;
        const uint32_t M = ow[Y * qw + wq];
        const uint32_t U = ow[yu * qw + wq], D = ow[yd * qw + wq];
        uint32_t L, R;
        if (p) {  // right neighbours: sites j+1..j+4
          L = M;
          R = __funnelshift_r(M, ow[Y * qw + (wq + 1 == qw ? 0 : wq + 1)], 8);
        } else {  // left neighbours: sites j-1..j+2
          L = __funnelshift_l(ow[Y * qw + (wq == 0 ? qw - 1 : wq - 1)], M, 8);
          R = M;
        }
        const uint32_t quad = (uint32_t)((row0 + r) >> 2);
        // bit set: the chain's site samples -1
        mw[q] = q == (int)threadIdx.x ? planes_decide_pre(L, R, U, D, MS, pre, gc0 >> 3, quad, sweep, keys)
                                      : planes_decide(L, R, U, D, MS, gc0 >> 3, quad, sweep, keys);
      }
    }
    for (int r = threadIdx.x; !PLANES && r < half_sites; r += blockDim.x) {
      const int Y = (int)fdiv((uint32_t)r, div_hw), j = r - Y * hw;
      const int p = (Y + c) & 1;
      const int jl = wrapi(j - 1 + p, hw), jr = wrapi(j + p, hw);
      const int yu = wrapi(Y - 1, H), yd = wrapi(Y + 1, H);
      const uint32_t N = (uint32_t)other[Y * hw + jl] | ((uint32_t)other[Y * hw + jr] << 8) |
                         ((uint32_t)other[yu * hw + j] << 16) | ((uint32_t)other[yd * hw + j] << 24);
      const uint32_t row = (uint32_t)(row0 + r);
      const u32x4 a = philox4x32_10(u32x4{gc0 >> 3, row, sweep, kSaltLatticeSpin}, keys);
      const uint32_t w[4] = {a.x, a.y, a.z, a.w};
      // transpose: byte v of (lo, hi) = chain v's pattern (bit k = neighbour k is -1)
      uint32_t lo = N, t;
      t = (lo ^ (lo >> 7)) & 0x00AA00AAu;
      lo = lo ^ t ^ (t << 7);
      t = (lo ^ (lo >> 14)) & 0x0000CCCCu;
      lo = lo ^ t ^ (t << 14);
      const uint32_t hi = (lo >> 4) & 0x0F0F0F0Fu;
      lo &= 0x0F0F0F0Fu;
      uint32_t down = 0u;
      int32_t d[8];  // threshold top bits - draw top bits: > 0 up, < 0 down, 0 tie
      bool tie = false;
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const uint32_t idx = __byte_perm(v < 4 ? lo : hi, 0u, 0x4440u + (v & 3));
        const int32_t h = (int32_t)((v & 1) ? (w[v >> 1] >> 16) : (w[v >> 1] & 0xFFFFu));
        d[v] = TH[idx] - h;
        down |= ((uint32_t)d[v] >> 31) << v;
        tie |= d[v] == 0;
      }
      if (tie) {  // rare: decide the tied chains on their refill bits
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          if (d[v] == 0) {
            const uint32_t idx = __byte_perm(v < 4 ? lo : hi, 0u, 0x4440u + (v & 3));
            const uint32_t f = philox4x32_10(u32x4{gc0 + v, row, sweep, kSaltLatticeRefill}, keys).x >> 25;
            if (f >= TL[idx]) down |= 1u << v;
          }
        }
      }
      mine[r] = (unsigned char)down;
    }
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(res_smem_u32(&half_bar)) : "memory");
    if (PLANES && t + 1 < n_half) eager_for(t + 1, pre);
    if (!failed && !res_bar_wait(&half_bar, (uint32_t)(t & 1))) {  // never expected: every thread arrives
      failed = true;  // later phases are not waited for; every thread still arrives and meets every barrier
      if (error) atomicExch(error, kErrHalfSweepWait);
    }
    if (t + 1 == next_obs) {  // per-chain magnetisation after this half-sweep
      if (threadIdx.x < 8) counts[threadIdx.x] = 0;
      __syncthreads();
      int local[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int i = threadIdx.x; i < 2 * half_sites; i += blockDim.x) {
        if (!((obs_colours >> (i / half_sites)) & 1)) continue;
        const uint32_t v8 = lat[i];
#pragma unroll
        for (int v = 0; v < 8; ++v) local[v] += (v8 >> v) & 1;
      }
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        int x = local[v];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        if ((threadIdx.x & 31) == 0) atomicAdd(&counts[v], x);
      }
      __syncthreads();
      if (threadIdx.x < 8) {
        const int n_sites = ((obs_colours & 1) ? half_sites : 0) + ((obs_colours & 2) ? half_sites : 0);
        obs[taken * C + 8 * g + threadIdx.x] = (double)(n_sites - 2 * counts[threadIdx.x]);
      }
      ++taken;
      next_obs = taken < n_obs ? next_obs + obs_every : -1;
      __syncthreads();
    }
  }
  // write back this group's byte of every row (other bytes of the word belong to other CTAs)
  for (int i = threadIdx.x; i < 2 * half_sites; i += blockDim.x) {
    const int c = i / half_sites, r = i - c * half_sites;
    const int64_t row = (c ? row0_c1 : row0_c0) + r;
    reinterpret_cast<unsigned char*>(state + row * words + word)[byte_in_word] = lat[i];
  }
}

}  // namespace
}  // namespace tthrml

namespace {
int resident_impl(uint32_t* state, int64_t n_chains, int32_t height, int32_t width, int64_t row0_colour0,
                  int64_t row0_colour1, const uint32_t* thresholds, uint64_t seed, uint32_t sweep0, int32_t colour0,
                  int64_t n_half_sweeps, double* obs, int64_t obs_first, int64_t obs_every, int64_t n_obs,
                  int32_t obs_colours, int64_t chain_offset, const tthrml_run_ctl* ctl, int32_t* error, void* stream,
                  bool planes) {
  using namespace tthrml;
  if (!state || !thresholds || height <= 0 || width <= 0 || height % 2 || width % 2 || n_chains <= 0 ||
      n_chains % 32 || chain_offset % 8 || (colour0 != 0 && colour0 != 1) || n_half_sweeps < 0) {
    set_error("tthrml_ising2d_resident: invalid arguments (even dimensions, n_chains %% 32 == 0, "
              "chain_offset %% 8 == 0)");
    return TTHRML_ERR_ARG;
  }
  if (obs && (n_obs <= 0 || obs_first < 1 || obs_every < 1 || obs_first + (n_obs - 1) * obs_every > n_half_sweeps ||
              obs_colours < 1 || obs_colours > 3)) {
    set_error("tthrml_ising2d_resident: observation schedule outside the run");
    return TTHRML_ERR_ARG;
  }
  const int64_t smem = (int64_t)height * width;  // both colours, one byte per site
  int dev = 0, max_smem = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return cuda_status(e, "tthrml_ising2d_resident: device query");
  if (smem + 256 > max_smem) {
    set_error("tthrml_ising2d_resident: a %d x %d lattice needs %lld bytes of shared memory per CTA (%d available)",
              (int)height, (int)width, (long long)smem, max_smem);
    return TTHRML_ERR_UNSUPPORTED;
  }
  if (planes && (width % 8 || row0_colour0 % 4 || row0_colour1 % 4)) {
    set_error("tthrml_ising2d_resident_planes: width %% 8 == 0 and block rows %% 4 == 0 required");
    return TTHRML_ERR_ARG;
  }
  auto kernel = planes ? k_ising2d_resident<true> : k_ising2d_resident<false>;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_status(e, "k_ising2d_resident shared memory attribute");
  if (n_half_sweeps == 0 && !obs) return TTHRML_OK;
  kernel<<<(unsigned)(n_chains / 8), kResThreads, (size_t)smem, (cudaStream_t)stream>>>(
      state, n_chains, height, width, row0_colour0, row0_colour1, thresholds, seed, sweep0, colour0, n_half_sweeps,
      obs, obs_first, obs_every, n_obs, obs_colours, chain_offset, ctl, error, make_fastdiv((uint32_t)(width / 2)));
  return launch_status("k_ising2d_resident launch");
}

}  // namespace

extern "C" int tthrml_ising2d_resident(uint32_t* state, int64_t n_chains, int32_t height, int32_t width,
                                       int64_t row0_colour0, int64_t row0_colour1, const uint32_t* thresholds,
                                       uint64_t seed, uint32_t sweep0, int32_t colour0, int64_t n_half_sweeps,
                                       double* obs, int64_t obs_first, int64_t obs_every, int64_t n_obs,
                                       int32_t obs_colours, int64_t chain_offset, const tthrml_run_ctl* ctl,
                                       int32_t* error, void* stream) {
  return resident_impl(state, n_chains, height, width, row0_colour0, row0_colour1, thresholds, seed, sweep0, colour0,
                       n_half_sweeps, obs, obs_first, obs_every, n_obs, obs_colours, chain_offset, ctl, error, stream,
                       false);
}

extern "C" int tthrml_ising2d_resident_planes(uint32_t* state, int64_t n_chains, int32_t height, int32_t width,
                                              int64_t row0_colour0, int64_t row0_colour1, const uint32_t* thresholds,
                                              uint64_t seed, uint32_t sweep0, int32_t colour0, int64_t n_half_sweeps,
                                              double* obs, int64_t obs_first, int64_t obs_every, int64_t n_obs,
                                              int32_t obs_colours, int64_t chain_offset, const tthrml_run_ctl* ctl,
                                              int32_t* error, void* stream) {
  return resident_impl(state, n_chains, height, width, row0_colour0, row0_colour1, thresholds, seed, sweep0, colour0,
                       n_half_sweeps, obs, obs_first, obs_every, n_obs, obs_colours, chain_offset, ctl, error, stream,
                       true);
}
