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
constexpr int kEpiWarps = 8;  // two per TMEM lane quadrant, each taking half of the columns
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
};

// Tile t of a persistent CTA -> (m block, n block): groups of kGroupM row
// blocks are walked n-fastest, so the tiles in flight at one time share a few
// A row panels and a band of B panels in L2.
constexpr int kGroupM = 16;
__device__ __forceinline__ void tile_coords(int t, int m_blocks, int n_blocks, int& mb, int& nb) {
  const int per_group = kGroupM * n_blocks;
  const int g = t / per_group, w = t - g * per_group;
  const int rows = min(kGroupM, m_blocks - g * kGroupM);
  mb = g * kGroupM + w % rows;
  nb = w / rows;
}

// Epilogue of one 32-column chunk of one row (chain m): draw and store.
template <int FAMILY, bool VARIATES>
__device__ __forceinline__ void draw_chunk(const DenseArgs& a, const float (&acc)[32], int64_t m, int64_t n_first,
                                           uint32_t sweep, uint32_t k0, uint32_t k1, float inv, float sd_g,
                                           int64_t vs) {
  const int64_t gchain = a.chain_offset + m;
  float outf[32];
  u32x4 r{0u, 0u, 0u, 0u};
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int64_t n = n_first + j;
    const int64_t row = a.row0 + n;
    const float field = a.bias ? __fadd_rn(acc[j], __ldg(a.bias + n)) : acc[j];
    float v;
    if (FAMILY == TTHRML_SPIN) {
      bool up;
      if (VARIATES) {
        up = __fmul_rn(2.0f, field) > __ldg(a.variates + (vs * a.N + n) * a.M + m);
      } else {
        if (j == 0 || (row & 3) == 0)
          r = philox4x32_10(u32x4{(uint32_t)gchain, (uint32_t)(row >> 2), sweep, kSaltDenseSpin}, k0, k1);
        up = spin_up_philox(field, word_of(r, (int)(row & 3)));
      }
      v = up ? 1.0f : -1.0f;
    } else {
      float xi;
      if (VARIATES) {
        xi = __ldg(a.variates + (vs * a.N + n) * a.M + m);
      } else {
        if (j == 0 || (row & 1) == 0)
          r = philox4x32_10(u32x4{(uint32_t)gchain, (uint32_t)(row >> 1), sweep, kSaltDenseGauss}, k0, k1);
        const int w = (int)(row & 1) * 2;
        xi = sqrtf(-2.0f * logf(uniform_open(word_of(r, w)))) * cospif(2.0f * uniform_open(word_of(r, w + 1)));
      }
      v = __fadd_rn(__fmul_rn(field, inv), __fmul_rn(sd_g, xi));
    }
    outf[j] = v;
  }
  if (a.out_f32) {
    float4* df = reinterpret_cast<float4*>(a.out_f32 + m * a.N + n_first);
#pragma unroll
    for (int q = 0; q < 8; ++q) df[q] = make_float4(outf[4 * q], outf[4 * q + 1], outf[4 * q + 2], outf[4 * q + 3]);
  }
  // piece p = bf16(v - pieces 0..p-1); each remainder is exact in float32, so
  // three pieces carry all 24 significand bits
  __nv_bfloat16* row = a.out + m * (a.N * a.pieces) + n_first;
  for (int p = 0; p < a.pieces; ++p) {
    __align__(16) __nv_bfloat16 outv[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      outv[j] = __float2bfloat16_rn(outf[j]);
      outf[j] = __fsub_rn(outf[j], __bfloat162float(outv[j]));
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
        tile_coords(t, m_blocks, n_blocks, mb, nb);
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
    const int half = (warp - 2) >> 2;
    int it = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
      int mb, nb;
      tile_coords(t, m_blocks, n_blocks, mb, nb);
      const int b = it & 1;
      const bool ok = mbar_wait(&acc_full[b], (uint32_t)(it >> 1) & 1u);
      if (!ok) {
        atomicExch(args.error, kErrAccWait);
        break;
      }
      tc_fence_after();
      const uint32_t sweep = args.sweep + (args.ctl ? args.ctl->sweep : 0u);
      const uint64_t sd = args.ctl ? args.ctl->seed : args.seed;
      const float inv = 1.0f / __fadd_rn(args.precision, 1e-6f);
      const float sd_g = sqrtf(inv);
      const int64_t vs =
          args.variates ? (int64_t)(sweep % (uint32_t)(args.variates_sweeps > 0 ? args.variates_sweeps : 1)) : 0;
      const int64_t m = (int64_t)mb * BM + quad * 32 + lane;
      for (int c = half; c < BN / 32; c += 2) {
        float acc[32];
        tmem_load32(tmem + (uint32_t)(b * kTmemCols) + ((uint32_t)(quad * 32) << 16) + (uint32_t)(c * 32), acc);
        draw_chunk<FAMILY, VARIATES>(args, acc, m, (int64_t)nb * BN + c * 32, sweep, seed_lo(sd), seed_hi(sd), inv,
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

}  // namespace
}  // namespace tthrml

extern "C" int tthrml_dense_field_sample(const void* source_state, const void* weights_nk, int64_t n_chains,
                                         int64_t n_units, int64_t n_sources, const float* bias, int32_t family,
                                         float precision, void* out_state, float* out_state_f32,
                                         int32_t out_pieces, int64_t row0,
                                         int64_t chain_offset, const float* variates, int64_t variates_sweeps,
                                         uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl, int32_t* error,
                                         void* stream) {
  using namespace tthrml;
  if (!source_state || !weights_nk || !out_state || !error) {
    set_error("tthrml_dense_field_sample: NULL argument");
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
      (out_state_f32 && ((uintptr_t)out_state_f32 % 16))) {
    set_error("tthrml_dense_field_sample: buffers must be 16-byte aligned and chain_offset a multiple of 4");
    return TTHRML_ERR_ARG;
  }
  CUtensorMap ma, mb;
  int rc = make_map(&ma, source_state, n_chains, n_sources, BM);
  if (rc) return rc;
  rc = make_map(&mb, weights_nk, n_units, n_sources, BN);
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
  int sms = 0, dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_status(e, "tthrml_dense_field_sample: device query");
  const int64_t n_tiles = (n_chains / BM) * (n_units / BN);
  const int grid = (int)(n_tiles < sms ? n_tiles : sms);
  cudaStream_t st = (cudaStream_t)stream;
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
  return launch_status("k_dense_field_sample launch");
}
