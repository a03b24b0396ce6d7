// Dense bipartite block update on the 5th-generation tensor cores (tcgen05).
//
// For a block whose sources are all the units of another block through a
// dense weight matrix (the visible/hidden blocks of an RBM), the field of every
// (chain, unit) is one entry of a GEMM over the chain batch:
//     field[m][n] = sum_k  S[m][k] * W[n][k]        (+ bias[n])
// with S the source block's state (chains x source units, bf16, row-major) and
// W the couplings stored target-major (units x source units, bf16, K-major).
// The new state of the target block is drawn in the epilogue straight from
// the TMEM accumulator: spin (+1 with probability sigmoid(2*gamma)) or gaussian
// (mean = field*var, var = 1/(precision + 1e-6); tt_thrml/compiler.py:321-365),
// and written back as bf16, the operand layout of the next GEMM.
//
// Kernel structure (persistent, one CTA per SM walking 128 x 256 output tiles,
// 10 warps):
//   warp 0 lane 0 : TMA producer, 4-stage ring of 128x64 A and 256x64 B bf16
//                   tiles in 128B-swizzled shared memory (full/empty mbarriers);
//   warp 1        : allocates 512 TMEM columns (two 128 x 256 fp32
//                   accumulators); lane 0 issues tcgen05.mma.kind::f16
//                   (M=128, N=256, K=16) and tcgen05.commit releases each stage
//                   and each finished accumulator;
//   warps 2..9    : epilogue, two per 32-lane TMEM quadrant (even / odd
//                   32-column chunks), tcgen05.ld, draw, store bf16 rows.
// Every wait is bounded by a clock limit; on expiry the kernel records an
// error code, drains its own copies and MMAs (bounded), frees TMEM and exits.
#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>

#include "common.cuh"

namespace tthrml {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KiB
constexpr int B_BYTES = BN * BK * 2;  // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
#ifndef TTHRML_DENSE_EPI_WARPS
#define TTHRML_DENSE_EPI_WARPS 8
#endif
// epilogue warps: kEpiGroups per TMEM lane quadrant, group g taking the 32-column chunks c = g mod kEpiGroups
constexpr int kEpiWarps = TTHRML_DENSE_EPI_WARPS;
constexpr int kEpiGroups = kEpiWarps / 4;
constexpr int kDenseThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t kTmemCols = 256;
constexpr int SMEM_BYTES = 1024 /*alignment slack*/ + STAGES * STAGE_BYTES + 256 /*barriers*/;
constexpr long long kWaitCycles = 4ll << 30;  // about two seconds at 2 GHz

enum : int { kErrNone = 0, kErrFullWait = 1, kErrEmptyWait = 2, kErrAccWait = 3 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase of `parity` to complete; false when the clock limit expires.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_test(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) return false;
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// UMMA shared-memory descriptor of a K-major tile in the 128B-swizzle layout
// written by TMA (rows of 128 B, 8-row groups 1024 B apart): start address,
// leading offset 16 B, stride offset 1024 B, descriptor version 1, layout 2.
__device__ __forceinline__ uint64_t umma_desc_sw128(const void* tile) {
  const uint64_t addr = (uint64_t)(smem_u32(tile) >> 4) & 0x3FFFull;
  return addr | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor: D fp32, A and B bf16, both K-major, N = BN, M = BM.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_load32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

struct DenseArgs {
  const float* bias;       // [N] or NULL
  __nv_bfloat16* out;      // [M][pieces * N] new target state: bf16 pieces, value = sum over pieces
  float* out_f32;          // [M][N] same values in float32, or NULL
  int32_t pieces;          // 1: bf16 value; 2-3: successive bf16 remainders (3 is exact for float32)
  const float* variates;   // [variates_sweeps][N][M] (unit-major, chains innermost) or NULL
  int64_t variates_sweeps;
  int64_t M, N, K;
  int64_t row0;            // flat state row of target unit 0 (Philox counter)
  int64_t chain_offset;
  uint64_t seed;
  uint32_t sweep;
  int32_t family;          // TTHRML_SPIN or TTHRML_GAUSSIAN
  float precision;         // gaussian: sum of precision contributions (1 for unit variance)
  const tthrml_run_ctl* ctl;
  int* error;              // device word, set on a wait timeout
  uint32_t* ties;          // near-threshold spin decisions: [count, blocks done, dropped, 0, (m, n) x ties_cap]
  int64_t ties_cap;        // or NULL: decisions from the float32 field alone
  int32_t group;           // CTA-pair kernel: row blocks per raster group
};

// A spin decision whose float32 margin is this close to the threshold (in units of u * (1 + e^(-2 gamma))
// around 1, or of 2 gamma - logit in variates mode; |t - 1| ~ (1 - u) |2 gamma - logit u|) is decided
// again from the exact field.  The tensor cores' float32 accumulation of a K-term field can be off by
// ~1e-5 at K = 4096 with terms of size 0.01; a decision the float32 field gets wrong at a true margin
// beyond the 1e-5 band therefore shows a float32 margin below (error - 1e-5), which this bound catches
// for errors up to 2e-5.  The exact field is bias + sum_k A[m][k] B[n][k] in double (bf16 products are
// exact there).  The epilogue only records such decisions (a few in 10^5); k_dense_settle, launched
// next on the same stream, decides them again and overwrites their outputs.
constexpr float kNearTie = 1e-5f;
#ifndef TTHRML_DENSE_FAST_TRIG
#define TTHRML_DENSE_FAST_TRIG 1  // Box-Muller angle through the hardware sine / cosine (0: sincospif)
#endif
#ifndef TTHRML_DENSE_F32X2
#define TTHRML_DENSE_F32X2 1  // spin draws with packed f32x2 arithmetic (0: scalar)
#endif
#ifndef TTHRML_DENSE_SETTLE
#define TTHRML_DENSE_SETTLE 2  // 0: no near-threshold check, 1: check only, 2: check and record
#endif
constexpr int kTieHeaderWords = 4;  // count, blocks of k_dense_settle done, entries dropped (cumulative), 0

// Appends the (chain m, unit n_first + j) of every bit j of each lane's `near` to the tie list: one
// atomic per warp, then each lane's entries at its prefix offset.  Entries past the capacity are
// dropped (their float32 decisions stand) and counted by k_dense_settle.  All 32 lanes call it.
__device__ __forceinline__ void record_ties(uint32_t* ties, int64_t cap, uint32_t near, int64_t m,
                                            int64_t n_first) {
  const int lane = threadIdx.x & 31;
  const uint32_t cnt = (uint32_t)__popc(near);
  uint32_t incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  uint32_t base = 0u;
  if (lane == 31) base = atomicAdd(ties, incl);
  base = __shfl_sync(0xffffffffu, base, 31);
  uint32_t idx = base + incl - cnt;
  uint2* entries = reinterpret_cast<uint2*>(ties + kTieHeaderWords);
  while (near) {
    const int j = __ffs(near) - 1;
    near &= near - 1u;
    if ((int64_t)idx < cap) entries[idx] = make_uint2((uint32_t)m, (uint32_t)(n_first + j));
    ++idx;
  }
}

// Tile t of a persistent CTA -> (m block, n block): the row blocks are taken
// `group` at a time and each group is walked row-fastest, so the tiles in
// flight at one time share one or two B column panels while the group's A
// row panels stay in L2 for the sweep over the group's columns.  The
// single-CTA kernel takes 16 row blocks of 128 rows; the CTA-pair kernel
// sizes its groups of 256-row blocks to about 32 MiB of A panels
// (group x 256 x K x 2 bytes), which measured lowest in DRAM bytes for both
// GEMMs of the 4096 x 8192 RBM (K = 4096: 16 blocks, K = 8192: 8 blocks;
// 64 MiB groups or a plain row-major walk re-read more).
constexpr int kGroupM = 16;
__device__ __forceinline__ void tile_coords(int t, int m_blocks, int n_blocks, int group, int& mb, int& nb) {
  const int per_group = group * n_blocks;
  const int g = t / per_group, w = t - g * per_group;
  const int rows = min(group, m_blocks - g * group);
  mb = g * group + w % rows;
  nb = w / rows;
}

// The 32 biases of a chunk (n_first % 32 == 0, bias 16-byte aligned): eight 16-byte loads, the same
// addresses in every lane; zeros without a bias.
__device__ __forceinline__ void load_bias32(const float* bias, int64_t n_first, float (&b)[32]) {
  if (!bias) {
#pragma unroll
    for (int j = 0; j < 32; ++j) b[j] = 0.0f;
    return;
  }
  const float4* bq = reinterpret_cast<const float4*>(bias + n_first);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 v = __ldg(bq + q);
    b[4 * q] = v.x;
    b[4 * q + 1] = v.y;
    b[4 * q + 2] = v.z;
    b[4 * q + 3] = v.w;
  }
}

// Spin epilogue of one 32-column chunk of row m: bit j of the result is set when unit n_first + j samples
// -1.  +1 with probability sigmoid(2 field): u * (1 + e^(-2 field)) < 1 with u = uniform_open of the
// unit's Philox word (u is built with ALU operations, bit for bit the same value), or 2 field > logit.
// `near` receives the decisions within kNearTie of their threshold.
template <bool VARIATES>
__device__ __forceinline__ uint32_t spin_chunk(const DenseArgs& a, const float (&acc)[32], int64_t m,
                                               int64_t n_first, uint32_t sweep, const PhiloxKeys& keys,
                                               int64_t vs, uint32_t& near) {
  const int64_t gchain = a.chain_offset + m;
  const int64_t r0 = a.row0 + n_first;
  uint32_t down = 0u;
  near = 0u;
  if (VARIATES) {
    float b[32];
    load_bias32(a.bias, n_first, b);
    const float* vrow = a.variates + (vs * a.N + n_first) * a.M + m;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float field = __fadd_rn(acc[j], b[j]);
      const float d = __fsub_rn(__fmul_rn(2.0f, field), __ldg(vrow + (int64_t)j * a.M));
      down |= (d > 0.0f ? 0u : 1u) << j;
      if (TTHRML_DENSE_SETTLE) near |= (fabsf(d) < kNearTie ? 1u : 0u) << j;
    }
  } else if ((r0 & 3) == 0) {  // the chunk starts a Philox counter: word j % 4 of counter r0 / 4 + j / 4
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const u32x4 r = philox4x32_10(u32x4{(uint32_t)gchain, (uint32_t)((r0 >> 2) + q), sweep, kSaltDenseSpin}, keys);
      const uint32_t w[4] = {r.x, r.y, r.z, r.w};
      const float4 bq = a.bias ? __ldg(reinterpret_cast<const float4*>(a.bias + n_first) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float b[4] = {bq.x, bq.y, bq.z, bq.w};
#if TTHRML_DENSE_F32X2
      // two units per packed instruction: t = u * (1 + 2^(-2 log2(e) field)), decided against 1
#pragma unroll
      for (int i = 0; i < 4; i += 2) {
        const int j = 4 * q + i;
        const float2 field = __fadd2_rn(make_float2(acc[j], acc[j + 1]), make_float2(b[i], b[i + 1]));
        const float2 x = __fmul2_rn(field, make_float2(-2.8853900817779268f, -2.8853900817779268f));
        float e0, e1;
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(x.x));
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(x.y));
        const float2 u = __fadd2_rn(make_float2(__uint_as_float(0x3F800000u | (w[i] >> 9)),
                                                __uint_as_float(0x3F800000u | (w[i + 1] >> 9))),
                                    make_float2(-0.99999994039535522461f, -0.99999994039535522461f));
        const float2 t = __fmul2_rn(u, __fadd2_rn(make_float2(e0, e1), make_float2(1.0f, 1.0f)));
        down |= ((t.x < 1.0f ? 0u : 1u) | (t.y < 1.0f ? 0u : 2u)) << j;
        if (TTHRML_DENSE_SETTLE) {
          const float2 d = __fadd2_rn(t, make_float2(-1.0f, -1.0f));
          near |= ((fabsf(d.x) < kNearTie ? 1u : 0u) | (fabsf(d.y) < kNearTie ? 2u : 0u)) << j;
        }
      }
#else
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = 4 * q + i;
        const float field = __fadd_rn(acc[j], b[i]);
        const float t = uniform_open_alu(w[i]) * (1.0f + __expf(-2.0f * field));
        down |= (t < 1.0f ? 0u : 1u) << j;
        if (TTHRML_DENSE_SETTLE) near |= (fabsf(t - 1.0f) < kNearTie ? 1u : 0u) << j;
      }
#endif
    }
  } else {
    float b[32];
    load_bias32(a.bias, n_first, b);
    u32x4 r{0u, 0u, 0u, 0u};
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int64_t row = r0 + j;
      if (j == 0 || (row & 3) == 0)
        r = philox4x32_10(u32x4{(uint32_t)gchain, (uint32_t)(row >> 2), sweep, kSaltDenseSpin}, keys);
      const float field = __fadd_rn(acc[j], b[j]);
      const float t = uniform_open_alu(word_of(r, (int)(row & 3))) * (1.0f + __expf(-2.0f * field));
      down |= (t < 1.0f ? 0u : 1u) << j;
      if (TTHRML_DENSE_SETTLE) near |= (fabsf(t - 1.0f) < kNearTie ? 1u : 0u) << j;
    }
  }
  return down;
}

// Box-Muller on words 2p, 2p+1 of a counter: the normals of rows 4j+2p (cosine) and 4j+2p+1 (sine).
__device__ __forceinline__ void box_muller_pair(uint32_t w0, uint32_t w1, float& xc, float& xs) {
  const float rad = sqrtf(-2.0f * logf(uniform_open(w0)));
  float sn, cs;
#if TTHRML_DENSE_FAST_TRIG
  // theta = 2 pi u1 = phi + pi with phi = 2 pi (u1 - 1/2) in (-pi, pi), where the hardware sine and cosine
  // are accurate to ~5e-7 absolute: cos theta = -cos phi, sin theta = -sin phi
  __sincosf(6.2831853071795865f * (uniform_open_alu(w1) - 0.5f), &sn, &cs);
  xc = -rad * cs;
  xs = -rad * sn;
#else
  sincospif(2.0f * uniform_open(w1), &sn, &cs);
  xc = rad * cs;
  xs = rad * sn;
#endif
}

// Gaussian epilogue of one 32-column chunk: field * var + sqrt(var) * xi, xi the unit's normal from the
// counter (chain, row / 4, sweep, "DGAU") (or the uploaded normal).
template <bool VARIATES>
__device__ __forceinline__ void gauss_chunk(const DenseArgs& a, const float (&acc)[32], int64_t m,
                                            int64_t n_first, uint32_t sweep, const PhiloxKeys& keys, float inv,
                                            float sd_g, int64_t vs, float (&outf)[32]) {
  float b[32];
  load_bias32(a.bias, n_first, b);
  const int64_t gchain = a.chain_offset + m;
  const int64_t r0 = a.row0 + n_first;
  float xi[32];
  if (VARIATES) {
    const float* vrow = a.variates + (vs * a.N + n_first) * a.M + m;
#pragma unroll
    for (int j = 0; j < 32; ++j) xi[j] = __ldg(vrow + (int64_t)j * a.M);
  } else if ((r0 & 3) == 0) {  // the chunk starts a counter: rows 4q..4q+3 of the chunk share counter q
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const u32x4 r = philox4x32_10(u32x4{(uint32_t)gchain, (uint32_t)((r0 >> 2) + q), sweep, kSaltDenseGauss}, keys);
      box_muller_pair(r.x, r.y, xi[4 * q], xi[4 * q + 1]);
      box_muller_pair(r.z, r.w, xi[4 * q + 2], xi[4 * q + 3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int64_t row = r0 + j;
      const u32x4 r = philox4x32_10(u32x4{(uint32_t)gchain, (uint32_t)(row >> 2), sweep, kSaltDenseGauss}, keys);
      const int w = (int)((row >> 1) & 1) * 2;
      float xc, xs;
      box_muller_pair(word_of(r, w), word_of(r, w + 1), xc, xs);
      xi[j] = (row & 1) ? xs : xc;
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float field = a.bias ? __fadd_rn(acc[j], b[j]) : acc[j];
    outf[j] = __fadd_rn(__fmul_rn(field, inv), __fmul_rn(sd_g, xi[j]));
  }
}

// Epilogue of one 32-column chunk of one row (chain m): draw and store.  The new value goes to the
// float32 copy (if any) and as `pieces` bf16 pieces: piece p = bf16(v - pieces 0..p-1), each remainder
// exact in float32, so three pieces carry all 24 significand bits.  A spin's +-1 is one bf16 piece
// (0x3F80 / 0xBF80) and zero remainders.
template <int FAMILY, bool VARIATES>
__device__ __forceinline__ void draw_chunk(const DenseArgs& a, const float (&acc)[32], int64_t m, int64_t n_first,
                                           uint32_t sweep, const PhiloxKeys& keys, float inv, float sd_g,
                                           int64_t vs) {
  __nv_bfloat16* row = a.out + m * (a.N * a.pieces) + n_first;
  if (FAMILY == TTHRML_SPIN) {
    uint32_t near;
    const uint32_t down = spin_chunk<VARIATES>(a, acc, m, n_first, sweep, keys, vs, near);
    if (TTHRML_DENSE_SETTLE == 2 && a.ties != nullptr &&
        __any_sync(0xffffffffu, near != 0u))  // rare: k_dense_settle decides these again from the exact field
      record_ties(a.ties, a.ties_cap, near, m, n_first);
    if (a.out_f32) {
      float4* df = reinterpret_cast<float4*>(a.out_f32 + m * a.N + n_first);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(0x3F800000u | (((down >> (4 * q + i)) & 1u) << 31));
        df[q] = make_float4(v[0], v[1], v[2], v[3]);
      }
    }
    uint32_t w[16];  // bf16 pairs (unit 2k in the low half)
#pragma unroll
    for (int k = 0; k < 16; ++k)
      w[k] = 0x3F803F80u | (((down >> (2 * k)) & 1u) << 15) | (((down >> (2 * k + 1)) & 1u) << 31);
    uint4* dst = reinterpret_cast<uint4*>(row);
#pragma unroll
    for (int q = 0; q < 4; ++q) dst[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    for (int p = 1; p < a.pieces; ++p) {
      uint4* z = reinterpret_cast<uint4*>(row + p * a.N);
#pragma unroll
      for (int q = 0; q < 4; ++q) z[q] = make_uint4(0u, 0u, 0u, 0u);
    }
    return;
  }
  float outf[32];
  gauss_chunk<VARIATES>(a, acc, m, n_first, sweep, keys, inv, sd_g, vs, outf);
  if (a.out_f32) {
    float4* df = reinterpret_cast<float4*>(a.out_f32 + m * a.N + n_first);
#pragma unroll
    for (int q = 0; q < 8; ++q) df[q] = make_float4(outf[4 * q], outf[4 * q + 1], outf[4 * q + 2], outf[4 * q + 3]);
  }
  for (int p = 0; p < a.pieces; ++p) {
    __align__(16) __nv_bfloat16 outv[32];
    const bool last = p + 1 == a.pieces;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      outv[j] = __float2bfloat16_rn(outf[j]);
      if (!last) outf[j] = __fsub_rn(outf[j], __bfloat162float(outv[j]));
    }
    uint4* dst = reinterpret_cast<uint4*>(row + p * a.N);
    const uint4* srcv = reinterpret_cast<const uint4*>(outv);
#pragma unroll
    for (int q = 0; q < 4; ++q) dst[q] = srcv[q];
  }
}

// Persistent kernel: one CTA per SM walks output tiles; two TMEM accumulators
// (2 x 256 columns) let the epilogue of one tile run under the main loop of
// the next.
template <int FAMILY, bool VARIATES>
__global__ void __launch_bounds__(kDenseThreads, 1)
    k_dense_field_sample(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         DenseArgs args) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_k = (int)(args.K / BK);
  const int m_blocks = (int)(args.M / BM), n_blocks = (int)(args.N / BN);
  const int n_tiles = m_blocks * n_blocks;

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(2 * kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);  // one arrival per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  int last_it[2] = {-1, -1};  // MMA thread: last tile iteration committed into each accumulator

  if (warp == 0) {
    if (lane == 0) {
      int64_t issued = 0;
      bool failed = false;
      for (int t = blockIdx.x; t < n_tiles && !failed; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, m_blocks, n_blocks, kGroupM, mb, nb);
        for (int kb = 0; kb < num_k; ++kb) {
          const int s = (int)(issued % STAGES);
          const uint32_t round = (uint32_t)(issued / STAGES);
          if (!mbar_wait(&empty[s], (round & 1u) ^ 1u)) {
            atomicExch(args.error, kErrEmptyWait);
            failed = true;
            break;
          }
          mbar_expect_tx(&full[s], STAGE_BYTES);
          unsigned char* a = tiles + s * STAGE_BYTES;
          // K blocks from the last to the first: with several bf16 pieces per source value ([hi | mid | lo]
          // along K) the small remainders are summed while the accumulator is still small, so the float32
          // rounding of the accumulation is that of the hi pieces alone
          const int kc = (num_k - 1 - kb) * BK;
          tma_load_2d(a, &map_a, &full[s], kc, mb * BM);
          tma_load_2d(a + A_BYTES, &map_b, &full[s], kc, nb * BN);
          ++issued;
        }
      }
      // the copies issued must land before the CTA can exit
      for (int64_t j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
        if (!mbar_wait(&full[j % STAGES], (uint32_t)(j / STAGES) & 1u)) atomicExch(args.error, kErrFullWait);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int64_t consumed = 0;
      int it = 0;
      bool failed = false;
      for (int t = blockIdx.x; t < n_tiles && !failed; t += gridDim.x, ++it) {
        const int b = it & 1;
        const uint32_t use = (uint32_t)(it >> 1);
        if (!mbar_wait(&acc_empty[b], (use & 1u) ^ 1u)) {  // epilogue done with this accumulator
          atomicExch(args.error, kErrAccWait);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * kTmemCols);
        for (int kb = 0; kb < num_k; ++kb) {
          const int s = (int)(consumed % STAGES);
          if (!mbar_wait(&full[s], (uint32_t)(consumed / STAGES) & 1u)) {
            atomicExch(args.error, kErrFullWait);
            failed = true;
            break;
          }
          tc_fence_after();
          const unsigned char* a = tiles + s * STAGE_BYTES;
          const uint64_t ad = umma_desc_sw128(a), bd = umma_desc_sw128(a + A_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)  // K = 16 per MMA: +32 B within the swizzle atom
            umma_bf16(d, ad + 2ull * kk, bd + 2ull * kk, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);  // stage reusable once these MMAs have read it
          ++consumed;
        }
        umma_commit(&acc_full[b]);  // accumulator b complete (tracks every MMA issued so far)
        last_it[b] = it;
      }
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 of the finished
    // accumulator; warps 2-5 take the even 32-column chunks, warps 6-9 the odd
    const int quad = warp & 3;
    const int grp = (warp - 2) >> 2;
    int it = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
      int mb, nb;
      tile_coords(t, m_blocks, n_blocks, kGroupM, mb, nb);
      const int b = it & 1;
      const bool ok = mbar_wait(&acc_full[b], (uint32_t)(it >> 1) & 1u);
      if (!ok) {
        atomicExch(args.error, kErrAccWait);
        break;
      }
      tc_fence_after();
      const uint32_t sweep = args.sweep + (args.ctl ? args.ctl->sweep : 0u);
      const uint64_t sd = args.ctl ? args.ctl->seed : args.seed;
      const PhiloxKeys keys = philox_keys(seed_lo(sd), seed_hi(sd));  // round keys, once per tile
      const float inv = 1.0f / __fadd_rn(args.precision, 1e-6f);
      const float sd_g = sqrtf(inv);
      const int64_t vs =
          args.variates ? (int64_t)(sweep % (uint32_t)(args.variates_sweeps > 0 ? args.variates_sweeps : 1)) : 0;
      const int64_t m = (int64_t)mb * BM + quad * 32 + lane;
      for (int c = grp; c < BN / 32; c += kEpiGroups) {
        float acc[32];
        tmem_load32(tmem + (uint32_t)(b * kTmemCols) + ((uint32_t)(quad * 32) << 16) + (uint32_t)(c * 32), acc);
        draw_chunk<FAMILY, VARIATES>(args, acc, m, (int64_t)nb * BN + c * 32, sweep, keys, inv,
                                     sd_g, vs);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acc_empty[b])) : "memory");
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // every MMA this CTA issued has completed before TMEM is freed: the last
    // commit of each accumulator tracks all earlier MMAs (bounded waits)
    if (lane == 0) {
      for (int b = 0; b < 2; ++b)
        if (last_it[b] >= 0) (void)mbar_wait(&acc_full[b], (uint32_t)(last_it[b] >> 1) & 1u);
    }
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// CTA-pair kernel (tcgen05 cta_group::2), for chain counts that are multiples
// of 256.  A cluster of two CTAs on two SMs computes 256 x 256 output tiles:
// CTA r holds rows 128r..128r+127 of the tile's A slice and units
// 128r..128r+127 of its B slice in its own shared memory, so a stage is 32 KiB
// per CTA (half the B bytes of the single-CTA kernel) and 6 stages fit.  The
// even CTA (the leader) issues every MMA (M = 256, N = 256, K = 16) over both
// CTAs' operands; the accumulator rows of CTA r land in CTA r's TMEM, which
// its own 8 epilogue warps drain exactly as in the single-CTA kernel.
// Synchronisation (the protocol of the sm100 2-SM pipelines):
//   full[s]   (leader only)  the leader's producer arrives with the stage's
//             bytes of both CTAs; both CTAs' TMA loads complete on it (their
//             mbarrier address with the CTA-rank bit cleared);
//   empty[s]  (each CTA)     the leader's tcgen05.commit multicasts to both;
//   acc_full  (each CTA)     likewise, once a tile's MMAs are done;
//   acc_empty (leader only)  every epilogue warp of both CTAs arrives (16).
// TMEM is allocated and freed pairwise (cta_group::2 by warp 1 of each CTA);
// a cluster barrier after barrier set-up and another before the free keep
// either CTA from signalling the other's uninitialised or exited memory.
// Every mbarrier wait is bounded as in the single-CTA kernel.
// ---------------------------------------------------------------------------
#ifndef TTHRML_DENSE_2SM
#define TTHRML_DENSE_2SM 1
#endif
#ifndef TTHRML_DENSE_STAGES2
#define TTHRML_DENSE_STAGES2 6
#endif
constexpr int BM2 = 128, BN2H = 128, STAGES2 = TTHRML_DENSE_STAGES2;
constexpr int A2_BYTES = BM2 * BK * 2;   // 16 KiB
constexpr int B2_BYTES = BN2H * BK * 2;  // 16 KiB
constexpr int STAGE2_BYTES = A2_BYTES + B2_BYTES;
constexpr int SMEM2_BYTES = 1024 + STAGES2 * STAGE2_BYTES + 256;
constexpr uint32_t kPeerMask = 0xFEFFFFFFu;  // clears the CTA-rank bit of a shared::cluster address
// Instruction descriptor of the pair MMA: D fp32, A and B bf16, K-major, N = 256, M = 256.
constexpr uint32_t kIdesc2 = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t n_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_leader, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar_leader), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(kIdesc2), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u),
      "r"(0u), "r"(0u));
}
// arrives (once all earlier MMAs of this thread are done) on the barrier at this offset in both CTAs
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)0x3)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_leader(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(smem_u32(bar) & kPeerMask) : "memory");
}

template <int FAMILY, bool VARIATES>
__global__ void __launch_bounds__(kDenseThreads, 1)
    k_dense_field_sample_pair(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                              DenseArgs args) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES2 * STAGE2_BYTES);
  uint64_t* empty = full + STAGES2;
  uint64_t* acc_full = empty + STAGES2;  // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int num_k = (int)(args.K / BK);
  const int m_blocks = (int)(args.M / (2 * BM2)), n_blocks = (int)(args.N / BN);
  const int n_tiles = m_blocks * n_blocks;
  const int first = (int)cluster_id_x(), step = (int)n_clusters_x();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kEpiWarps);  // every epilogue warp of both CTAs
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(2 * kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers exist before either signals the other
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  int last_it[2] = {-1, -1};

  if (warp == 0) {
    if (lane == 0) {  // producer (both CTAs): this CTA's halves of the A and B slices
      int64_t issued = 0;
      bool failed = false;
      for (int t = first; t < n_tiles && !failed; t += step) {
        int mb, nb;
        tile_coords(t, m_blocks, n_blocks, args.group, mb, nb);
        for (int kb = 0; kb < num_k; ++kb) {
          const int s = (int)(issued % STAGES2);
          const uint32_t round = (uint32_t)(issued / STAGES2);
          if (!mbar_wait(&empty[s], (round & 1u) ^ 1u)) {
            atomicExch(args.error, kErrEmptyWait);
            failed = true;
            break;
          }
          if (leader) mbar_expect_tx(&full[s], 2 * STAGE2_BYTES);  // the stage's bytes of both CTAs
          unsigned char* a = tiles + s * STAGE2_BYTES;
          const int kc = (num_k - 1 - kb) * BK;  // K blocks last to first (see the single-CTA kernel)
          const uint32_t bar = smem_u32(&full[s]) & kPeerMask;
          tma_load_2d_pair(a, &map_a, bar, kc, mb * 2 * BM2 + (int)rank * BM2);
          tma_load_2d_pair(a + A2_BYTES, &map_b, bar, kc, nb * BN + (int)rank * BN2H);
          ++issued;
        }
      }
      // every stage this CTA filled has been consumed (released by the leader's MMAs) before exit
      for (int64_t j = issued > STAGES2 ? issued - STAGES2 : 0; j < issued; ++j)
        if (!mbar_wait(&empty[j % STAGES2], (uint32_t)(j / STAGES2) & 1u)) atomicExch(args.error, kErrEmptyWait);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // MMA issue: the leader only
      int64_t consumed = 0;
      int it = 0;
      bool failed = false;
      for (int t = first; t < n_tiles && !failed; t += step, ++it) {
        const int b = it & 1;
        const uint32_t use = (uint32_t)(it >> 1);
        if (!mbar_wait(&acc_empty[b], (use & 1u) ^ 1u)) {
          atomicExch(args.error, kErrAccWait);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * kTmemCols);
        for (int kb = 0; kb < num_k; ++kb) {
          const int s = (int)(consumed % STAGES2);
          if (!mbar_wait(&full[s], (uint32_t)(consumed / STAGES2) & 1u)) {
            atomicExch(args.error, kErrFullWait);
            failed = true;
            break;
          }
          tc_fence_after();
          const unsigned char* a = tiles + s * STAGE2_BYTES;
          const uint64_t ad = umma_desc_sw128(a), bd = umma_desc_sw128(a + A2_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_bf16_pair(d, ad + 2ull * kk, bd + 2ull * kk, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit_pair(&empty[s]);  // the stage is free again in both CTAs
          ++consumed;
        }
        umma_commit_pair(&acc_full[b]);  // both CTAs' accumulator halves complete
        last_it[b] = it;
      }
    }
  } else {
    // epilogue (both CTAs): this CTA's 128 rows of the tile, as in the single-CTA kernel
    const int quad = warp & 3;
    const int grp = (warp - 2) >> 2;
    int it = 0;
    for (int t = first; t < n_tiles; t += step, ++it) {
      int mb, nb;
      tile_coords(t, m_blocks, n_blocks, args.group, mb, nb);
      const int b = it & 1;
      if (!mbar_wait(&acc_full[b], (uint32_t)(it >> 1) & 1u)) {
        atomicExch(args.error, kErrAccWait);
        break;
      }
      tc_fence_after();
      const uint32_t sweep = args.sweep + (args.ctl ? args.ctl->sweep : 0u);
      const uint64_t sd = args.ctl ? args.ctl->seed : args.seed;
      const PhiloxKeys keys = philox_keys(seed_lo(sd), seed_hi(sd));  // round keys, once per tile
      const float inv = 1.0f / __fadd_rn(args.precision, 1e-6f);
      const float sd_g = sqrtf(inv);
      const int64_t vs =
          args.variates ? (int64_t)(sweep % (uint32_t)(args.variates_sweeps > 0 ? args.variates_sweeps : 1)) : 0;
      const int64_t m = (int64_t)mb * 2 * BM2 + (int64_t)rank * BM2 + quad * 32 + lane;
      for (int c = grp; c < BN / 32; c += kEpiGroups) {
        float acc[32];
        tmem_load32(tmem + (uint32_t)(b * kTmemCols) + ((uint32_t)(quad * 32) << 16) + (uint32_t)(c * 32), acc);
        draw_chunk<FAMILY, VARIATES>(args, acc, m, (int64_t)nb * BN + c * 32, sweep, keys, inv,
                                     sd_g, vs);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_leader(&acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1 && leader) {
    // every MMA the pair issued has completed (in both CTAs' TMEM) before TMEM is freed
    if (lane == 0) {
      for (int b = 0; b < 2; ++b)
        if (last_it[b] >= 0) (void)mbar_wait(&acc_full[b], (uint32_t)(last_it[b] >> 1) & 1u);
    }
    __syncwarp();
  }
  tc_fence_before();
  cluster_sync_all();  // neither CTA frees TMEM or exits while the other may still signal it
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kTmemCols));
}

// --- host side --------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_fn(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p) {
      set_error("cuTensorMapEncodeTiled is unavailable (%s)", cudaGetErrorString(e));
      return TTHRML_ERR_CUDA;
    }
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  *out = fn;
  return TTHRML_OK;
}

// Tensor map of a row-major bf16 matrix [rows][cols] read in (box_rows x 64) tiles, 128B swizzle.
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, uint32_t box_rows) {
  EncodeTiledFn fn;
  int rc = encode_fn(&fn);
  if (rc) return rc;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for a %lld x %lld bf16 matrix", (int)r, (long long)rows,
              (long long)cols);
    return TTHRML_ERR_CUDA;
  }
  return TTHRML_OK;
}

// Launches the CTA-pair kernel: clusters of 2 CTAs, as many as can be resident at once (persistent).
// ---------------------------------------------------------------------------
// Near-threshold settling.  One warp per recorded (chain m, unit n): the exact
// field bias[n] + sum_k A[m][k] B[n][k] in double (a bf16 product is exact in
// double; 8 terms per lane per step from 16-byte loads, rows 128-byte aligned
// because K % 64 == 0), the same variate as the epilogue (Philox word or
// uploaded logit) in double, and the decision written over the epilogue's:
// +-1 in piece 0, 0 in the remainder pieces, +-1 in the float32 copy.  The
// last block to finish clears the count, so the list is empty for the next
// launch on the stream (CUDA graph replays included).
// ---------------------------------------------------------------------------
struct SettleArgs {
  const __nv_bfloat16* a_mat;  // [M][K] source state
  const __nv_bfloat16* b_mat;  // [N][K] weights
  const float* bias;
  const float* variates;
  int64_t variates_sweeps;
  __nv_bfloat16* out;
  float* out_f32;
  int32_t pieces;
  int64_t M, N, K, row0, chain_offset;
  uint64_t seed;
  uint32_t sweep;
  const tthrml_run_ctl* ctl;
  uint32_t* ties;
  int64_t cap;
};

constexpr int kSettleThreads = 256;

template <bool VARIATES>
__global__ void __launch_bounds__(kSettleThreads) k_dense_settle(SettleArgs a) {
  const int lane = threadIdx.x & 31;
  const uint32_t count = *reinterpret_cast<volatile const uint32_t*>(a.ties);
  const int64_t n_entries = (int64_t)count < a.cap ? (int64_t)count : a.cap;
  const uint32_t sweep = a.sweep + (a.ctl ? a.ctl->sweep : 0u);
  const uint64_t sd = a.ctl ? a.ctl->seed : a.seed;
  const int64_t vs =
      a.variates ? (int64_t)(sweep % (uint32_t)(a.variates_sweeps > 0 ? a.variates_sweeps : 1)) : 0;
  const uint2* entries = reinterpret_cast<const uint2*>(a.ties + kTieHeaderWords);
  const int64_t warps = (int64_t)gridDim.x * (kSettleThreads / 32);
  for (int64_t i = (int64_t)blockIdx.x * (kSettleThreads / 32) + (threadIdx.x >> 5); i < n_entries; i += warps) {
    const uint2 e = entries[i];
    const int64_t m = e.x, n = e.y;
    if (m >= a.M || n >= a.N) continue;  // never recorded so; keeps every access below in bounds
    const __nv_bfloat16* ar = a.a_mat + m * a.K;
    const __nv_bfloat16* br = a.b_mat + n * a.K;
    double part[4] = {0.0, 0.0, 0.0, 0.0};  // four independent chains of double adds
#pragma unroll 8
    for (int64_t k = 8 * lane; k < a.K; k += 256) {
      const uint4 av = __ldg(reinterpret_cast<const uint4*>(ar + k));
      const uint4 bv = __ldg(reinterpret_cast<const uint4*>(br + k));
      const uint32_t aw[4] = {av.x, av.y, av.z, av.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        part[q] += (double)__uint_as_float(aw[q] << 16) * (double)__uint_as_float(bw[q] << 16);
        part[q] += (double)__uint_as_float(aw[q] & 0xFFFF0000u) * (double)__uint_as_float(bw[q] & 0xFFFF0000u);
      }
    }
    double acc = (part[0] + part[1]) + (part[2] + part[3]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      const double field = acc + (a.bias ? (double)__ldg(a.bias + n) : 0.0);
      double l;
      if (VARIATES) {
        l = (double)__ldg(a.variates + (vs * a.N + n) * a.M + m);
      } else {
        const int64_t row = a.row0 + n;
        const u32x4 r = philox4x32_10(u32x4{(uint32_t)(a.chain_offset + m), (uint32_t)(row >> 2), sweep,
                                            kSaltDenseSpin},
                                      seed_lo(sd), seed_hi(sd));
        const double u = (double)uniform_open(word_of(r, (int)(row & 3)));
        l = log(u) - log1p(-u);
      }
      const float v = 2.0 * field > l ? 1.0f : -1.0f;
      __nv_bfloat16* o = a.out + m * (a.N * a.pieces) + n;
      o[0] = __float2bfloat16_rn(v);
      for (int p = 1; p < a.pieces; ++p) o[p * a.N] = __float2bfloat16_rn(0.0f);
      if (a.out_f32) a.out_f32[m * a.N + n] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0 && (int64_t)count > a.cap) atomicAdd(a.ties + 2, count - (uint32_t)a.cap);
    __threadfence();
    if (atomicAdd(a.ties + 1, 1u) == gridDim.x - 1) {  // every block has read the count
      a.ties[0] = 0u;
      a.ties[1] = 0u;
    }
  }
}

int launch_settle(const DenseArgs& d, const void* a_mat, const void* b_mat, int sms, cudaStream_t st) {
  SettleArgs s;
  s.a_mat = reinterpret_cast<const __nv_bfloat16*>(a_mat);
  s.b_mat = reinterpret_cast<const __nv_bfloat16*>(b_mat);
  s.bias = d.bias;
  s.variates = d.variates;
  s.variates_sweeps = d.variates_sweeps;
  s.out = d.out;
  s.out_f32 = d.out_f32;
  s.pieces = d.pieces;
  s.M = d.M;
  s.N = d.N;
  s.K = d.K;
  s.row0 = d.row0;
  s.chain_offset = d.chain_offset;
  s.seed = d.seed;
  s.sweep = d.sweep;
  s.ctl = d.ctl;
  s.ties = d.ties;
  s.cap = d.ties_cap;
  const int64_t per_block = kSettleThreads / 32;
  const int64_t want = (d.ties_cap + per_block - 1) / per_block;
  const int grid = (int)(want < 2 * sms ? want : 2 * sms);
  if (d.variates)
    k_dense_settle<true><<<grid, kSettleThreads, 0, st>>>(s);
  else
    k_dense_settle<false><<<grid, kSettleThreads, 0, st>>>(s);
  return launch_status("k_dense_settle launch");
}

int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const DenseArgs& a, int32_t family, bool variates,
                cudaStream_t st) {
  const void* fn = family == TTHRML_SPIN
                       ? (variates ? (const void*)k_dense_field_sample_pair<TTHRML_SPIN, true>
                                   : (const void*)k_dense_field_sample_pair<TTHRML_SPIN, false>)
                       : (variates ? (const void*)k_dense_field_sample_pair<TTHRML_GAUSSIAN, true>
                                   : (const void*)k_dense_field_sample_pair<TTHRML_GAUSSIAN, false>);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kDenseThreads, 1, 1);
  cfg.dynamicSmemBytes = SMEM2_BYTES;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int64_t n_tiles = (a.M / (2 * BM2)) * (a.N / BN);
  int clusters = 0;
  cfg.gridDim = dim3(2, 1, 1);
  cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg);
  if (e != cudaSuccess) return cuda_status(e, "k_dense_field_sample_pair: cudaOccupancyMaxActiveClusters");
  if (clusters < 1) {
    set_error("k_dense_field_sample_pair: no CTA pair fits on this device");
    return TTHRML_ERR_UNSUPPORTED;
  }
  const int64_t want = n_tiles < clusters ? n_tiles : clusters;
  cfg.gridDim = dim3((unsigned)(2 * want), 1, 1);
  void* params[3] = {(void*)&ma, (void*)&mb, (void*)&a};
  e = cudaLaunchKernelExC(&cfg, fn, params);
  if (e != cudaSuccess) return cuda_status(e, "k_dense_field_sample_pair launch");
  return launch_status("k_dense_field_sample_pair launch");
}

}  // namespace
}  // namespace tthrml

namespace {

int dense_field_sample(const void* source_state, const void* weights_nk, int64_t n_chains, int64_t n_units,
                       int64_t n_sources, const float* bias, int32_t family, float precision, void* out_state,
                       float* out_state_f32, int32_t out_pieces, int64_t row0, int64_t chain_offset,
                       const float* variates, int64_t variates_sweeps, uint64_t seed, uint32_t sweep,
                       const tthrml_run_ctl* ctl, int32_t* error, uint32_t* ties, int64_t ties_capacity,
                       void* stream) {
  using namespace tthrml;
  if (!source_state || !weights_nk || !out_state || !error) {
    set_error("tthrml_dense_field_sample: NULL argument");
    return TTHRML_ERR_ARG;
  }
  if (ties && (ties_capacity < 1 || ties_capacity > 0x7fffffff || ((uintptr_t)ties % 16) ||
               n_units > 0xffffffffLL)) {  // entries hold 32-bit unit indices
    set_error("tthrml_dense_field_sample_ties: ties must be 16-byte aligned with 1 <= capacity < 2^31 and "
              "n_units < 2^32 (got capacity %lld, n_units %lld)", (long long)ties_capacity, (long long)n_units);
    return TTHRML_ERR_ARG;
  }
  if (n_chains <= 0 || n_units <= 0 || n_sources <= 0 || n_chains % BM || n_units % BN || n_sources % BK) {
    set_error("tthrml_dense_field_sample: chains must be a multiple of %d, units of %d and sources of %d "
              "(got %lld, %lld, %lld)", BM, BN, BK, (long long)n_chains, (long long)n_units, (long long)n_sources);
    return TTHRML_ERR_ARG;
  }
  if (n_chains / BM > 65535 || n_units / BN > 0x7fffffff || n_sources > 0x7fffffff || n_chains > 0x7fffffff) {
    set_error("tthrml_dense_field_sample: sizes exceed the launch grid");
    return TTHRML_ERR_ARG;
  }
  if (family != TTHRML_SPIN && family != TTHRML_GAUSSIAN) {
    set_error("tthrml_dense_field_sample: family must be spin or gaussian");
    return TTHRML_ERR_ARG;
  }
  if (out_pieces < 1 || out_pieces > 3) {
    set_error("tthrml_dense_field_sample: out_pieces must be 1, 2 or 3 (got %d)", (int)out_pieces);
    return TTHRML_ERR_ARG;
  }
  if (chain_offset % 4 || ((uintptr_t)source_state % 16) || ((uintptr_t)weights_nk % 16) || ((uintptr_t)out_state % 16) ||
      (out_state_f32 && ((uintptr_t)out_state_f32 % 16)) || (bias && ((uintptr_t)bias % 16))) {
    set_error("tthrml_dense_field_sample: buffers must be 16-byte aligned and chain_offset a multiple of 4");
    return TTHRML_ERR_ARG;
  }
  const bool pair = TTHRML_DENSE_2SM && n_chains % (2 * BM2) == 0;  // CTA-pair kernel: 256-row tiles
  CUtensorMap ma, mb;
  int rc = make_map(&ma, source_state, n_chains, n_sources, BM);
  if (rc) return rc;
  rc = make_map(&mb, weights_nk, n_units, n_sources, pair ? BN2H : BN);
  if (rc) return rc;
  {  // the shared-memory limit is a per-device function attribute
    static std::mutex mu;
    static bool attr_set[256] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
    if (dev < 0 || dev >= 256) {
      set_error("tthrml_dense_field_sample: device ordinal %d out of range", dev);
      return TTHRML_ERR_UNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev]) {
      const void* fns[4] = {(const void*)k_dense_field_sample<TTHRML_SPIN, false>,
                            (const void*)k_dense_field_sample<TTHRML_SPIN, true>,
                            (const void*)k_dense_field_sample<TTHRML_GAUSSIAN, false>,
                            (const void*)k_dense_field_sample<TTHRML_GAUSSIAN, true>};
      for (const void* f : fns) {
        e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return cuda_status(e, "k_dense_field_sample shared memory attribute");
      }
      const void* fns2[4] = {(const void*)k_dense_field_sample_pair<TTHRML_SPIN, false>,
                             (const void*)k_dense_field_sample_pair<TTHRML_SPIN, true>,
                             (const void*)k_dense_field_sample_pair<TTHRML_GAUSSIAN, false>,
                             (const void*)k_dense_field_sample_pair<TTHRML_GAUSSIAN, true>};
      for (const void* f : fns2) {
        e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES);
        if (e != cudaSuccess) return cuda_status(e, "k_dense_field_sample_pair shared memory attribute");
      }
      attr_set[dev] = true;
    }
  }
  DenseArgs a;
  a.bias = bias;
  a.out = reinterpret_cast<__nv_bfloat16*>(out_state);
  a.out_f32 = out_state_f32;
  a.pieces = out_pieces;
  a.variates = variates;
  a.variates_sweeps = variates_sweeps;
  a.M = n_chains;
  a.N = n_units;
  a.K = n_sources;
  a.row0 = row0;
  a.chain_offset = chain_offset;
  a.seed = seed;
  a.sweep = sweep;
  a.family = family;
  a.precision = precision;
  a.ctl = ctl;
  a.error = error;
  {  // raster groups of about 32 MiB of A panels (256-row blocks)
    const int64_t g = ((int64_t)32 << 20) / (2 * BM2 * n_sources * 2);
    const int64_t mblk = n_chains / (2 * BM2);
    a.group = (int32_t)(g < 1 ? 1 : (g > mblk ? (mblk > 0 ? mblk : 1) : g));
  }
  const bool settle = TTHRML_DENSE_SETTLE == 2 && ties != nullptr && family == TTHRML_SPIN;
  a.ties = settle ? ties : nullptr;
  a.ties_cap = settle ? ties_capacity : 0;
  int sms = 0, dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_status(e, "tthrml_dense_field_sample: device query");
  cudaStream_t st = (cudaStream_t)stream;
  if (pair) {
    rc = launch_pair(ma, mb, a, family, variates != nullptr, st);
    if (rc == TTHRML_OK && settle) rc = launch_settle(a, source_state, weights_nk, sms, st);
    return rc;
  }
  const int64_t n_tiles = (n_chains / BM) * (n_units / BN);
  const int grid = (int)(n_tiles < sms ? n_tiles : sms);
  if (family == TTHRML_SPIN) {
    if (variates)
      k_dense_field_sample<TTHRML_SPIN, true><<<grid, kDenseThreads, SMEM_BYTES, st>>>(ma, mb, a);
    else
      k_dense_field_sample<TTHRML_SPIN, false><<<grid, kDenseThreads, SMEM_BYTES, st>>>(ma, mb, a);
  } else {
    if (variates)
      k_dense_field_sample<TTHRML_GAUSSIAN, true><<<grid, kDenseThreads, SMEM_BYTES, st>>>(ma, mb, a);
    else
      k_dense_field_sample<TTHRML_GAUSSIAN, false><<<grid, kDenseThreads, SMEM_BYTES, st>>>(ma, mb, a);
  }
  rc = launch_status("k_dense_field_sample launch");
  if (rc == TTHRML_OK && settle) rc = launch_settle(a, source_state, weights_nk, sms, st);
  return rc;
}

}  // namespace

extern "C" int tthrml_dense_field_sample(const void* source_state, const void* weights_nk, int64_t n_chains,
                                         int64_t n_units, int64_t n_sources, const float* bias, int32_t family,
                                         float precision, void* out_state, float* out_state_f32,
                                         int32_t out_pieces, int64_t row0,
                                         int64_t chain_offset, const float* variates, int64_t variates_sweeps,
                                         uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl, int32_t* error,
                                         void* stream) {
  return dense_field_sample(source_state, weights_nk, n_chains, n_units, n_sources, bias, family, precision,
                            out_state, out_state_f32, out_pieces, row0, chain_offset, variates, variates_sweeps,
                            seed, sweep, ctl, error, nullptr, 0, stream);
}

extern "C" int tthrml_dense_field_sample_ties(const void* source_state, const void* weights_nk, int64_t n_chains,
                                              int64_t n_units, int64_t n_sources, const float* bias, int32_t family,
                                              float precision, void* out_state, float* out_state_f32,
                                              int32_t out_pieces, int64_t row0, int64_t chain_offset,
                                              const float* variates, int64_t variates_sweeps, uint64_t seed,
                                              uint32_t sweep, const tthrml_run_ctl* ctl, int32_t* error,
                                              uint32_t* ties, int64_t ties_capacity, void* stream) {
  if (!ties) {
    tthrml::set_error("tthrml_dense_field_sample_ties: NULL tie list");
    return TTHRML_ERR_ARG;
  }
  return dense_field_sample(source_state, weights_nk, n_chains, n_units, n_sources, bias, family, precision,
                            out_state, out_state_f32, out_pieces, row0, chain_offset, variates, variates_sweeps,
                            seed, sweep, ctl, error, ties, ties_capacity, stream);
}
