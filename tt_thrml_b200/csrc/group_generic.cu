// Generic group kernel: any mix of spin / categorical / gaussian blocks over
// ragged-ELL interaction tables, one thread per (row, chain), chain fastest so
// a warp reads one contiguous state row per gathered source.
//
// Math follows the reference group kernel term for term
// (tt_thrml/compiler.py:274-385): per interaction the terms are summed in
// order starting from the first, interaction contributions are added in
// program order, categorical sources select a weight slice, non-categorical
// sources multiply.  Explicit __fmul_rn/__fadd_rn keep the compiler from
// contracting products into FMAs so results match a plain float32 evaluation.
#include "common.cuh"

namespace tthrml {
namespace {

template <typename T>
__device__ __forceinline__ float load_state(const T* s, int64_t i) {
  return (float)s[i];
}

template <typename T>
__device__ __forceinline__ void store_value(T* s, int64_t i, float v);
template <>
__device__ __forceinline__ void store_value<float>(float* s, int64_t i, float v) {
  s[i] = v;
}
template <>
__device__ __forceinline__ void store_value<int8_t>(int8_t* s, int64_t i, float v) {
  s[i] = (int8_t)__float2int_rn(v);
}

// Weight offset selected by the categorical sources of term e (row-major over
// the categorical axes, tt_thrml/compiler.py:289-300).  Returns -1 when a
// source holds a value outside [0, q): its one-hot row is all zero in the
// reference, so the selected weight is 0.
template <typename T>
__device__ __forceinline__ int64_t cat_select(const tthrml_interaction& it, const T* state,
                                              int64_t C, int64_t chain, int64_t e) {
  int64_t sel = 0;
  const int first = it.n_sources - it.n_categorical;
  for (int j = 0; j < it.n_categorical; ++j) {
    const int32_t src = it.sources[(int64_t)(first + j) * it.nnz + e];
    const float v = load_state(state, (int64_t)src * C + chain);
    const int q = it.cat_q[j];
    const int k = (int)v;
    if (!(v == (float)k) || k < 0 || k >= q) return -1;
    sel = sel * q + k;
  }
  return sel;
}

// Product of the non-categorical sources of term e (tt_thrml/compiler.py:274-286).
template <typename T>
__device__ __forceinline__ float source_scale(const tthrml_interaction& it, const T* state,
                                              int64_t C, int64_t chain, int64_t e) {
  const int n_mult = it.n_sources - it.n_categorical;
  float s = load_state(state, (int64_t)it.sources[e] * C + chain);
  for (int j = 1; j < n_mult; ++j)
    s = __fmul_rn(s, load_state(state, (int64_t)it.sources[(int64_t)j * it.nnz + e] * C + chain));
  return s;
}

// Scalar field of one node for spin / gaussian targets: sum over the
// interactions whose kind matches `want_precision` (tt_thrml/compiler.py:303-318).
template <typename T>
__device__ float scalar_field(const tthrml_block& B, int want_precision, const T* state, int64_t C,
                              int64_t chain, int64_t i, bool* any) {
  float gamma = 0.0f;
  *any = false;
  for (int k = 0; k < B.n_interactions; ++k) {
    const tthrml_interaction& it = B.interactions[k];
    if ((it.kind == TTHRML_KIND_PRECISION) != (want_precision != 0)) continue;
    const int64_t e0 = it.row_ptr[i], e1 = it.row_ptr[i + 1];
    const int n_mult = it.n_sources - it.n_categorical;
    const int64_t cat_stride = it.w_inner;  // q_target == 1 here
    float contrib = 0.0f;
    bool first = true;
    for (int64_t e = e0; e < e1; ++e) {
      float w = 0.0f;
      if (it.n_categorical) {
        const int64_t sel = cat_select(it, state, C, chain, e);
        w = sel < 0 ? 0.0f : it.weights[e * cat_stride + sel];
      } else {
        w = it.weights[e * cat_stride];
      }
      const float term = n_mult ? __fmul_rn(w, source_scale(it, state, C, chain, e)) : w;
      contrib = first ? term : __fadd_rn(contrib, term);
      first = false;
    }
    gamma = *any ? __fadd_rn(gamma, contrib) : contrib;
    *any = true;
  }
  return gamma;
}

template <typename T, bool VARIATES>
__global__ void __launch_bounds__(256) k_group_generic(tthrml_group g) {
  const int64_t C = g.n_chains;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (tid >= g.group_rows * C) return;
  const int64_t lrow = tid / C;
  const int64_t chain = tid - lrow * C;

  int b = 0;
  int64_t base = 0;
  while (b + 1 < g.n_blocks && lrow >= base + g.blocks[b].n_nodes) {
    base += g.blocks[b].n_nodes;
    ++b;
  }
  const tthrml_block& B = g.blocks[b];
  const int64_t i = lrow - base;
  const int64_t row = B.row_start + i;
  const T* state = (const T*)g.state;
  T* out = g.in_place ? (T*)g.state : (T*)g.scratch;
  const int64_t out_idx = (g.in_place ? row : lrow) * C + chain;
  const int64_t gchain = g.chain_offset + chain;
  const uint64_t seed = g.ctl ? g.ctl->seed : g.seed;
  const uint32_t k0 = seed_lo(seed), k1 = seed_hi(seed);
  const uint32_t sweep = g.sweep + (g.ctl ? g.ctl->sweep : 0u);
  // variates hold variates_sweeps sweeps; the host never runs past them, the
  // modulo only keeps a misuse in bounds
  const int64_t vsweep = VARIATES ? (int64_t)(sweep % (uint32_t)(B.variates_sweeps > 0 ? B.variates_sweeps : 1)) : 0;

  if (B.family == TTHRML_SPIN) {
    bool any;
    const float gamma = scalar_field(B, 0, state, C, chain, i, &any);
    bool up;
    if (VARIATES) {
      const float l = B.variates[(vsweep * B.n_nodes + i) * C + chain];
      up = __fmul_rn(2.0f, gamma) > l;
    } else {
      const u32x4 r = philox4x32_10(u32x4{(uint32_t)(gchain >> 2), (uint32_t)row, sweep, kSaltSpin}, k0, k1);
      up = spin_up_philox(gamma, word_of(r, (int)(gchain & 3)));
    }
    store_value(out, out_idx, up ? 1.0f : -1.0f);
  } else if (B.family == TTHRML_CATEGORICAL) {
    const int q = B.n_categories;
    float theta[TTHRML_MAX_CATEGORIES];
    bool seen = false;
    for (int k = 0; k < q; ++k) theta[k] = 0.0f;
    for (int n = 0; n < B.n_interactions; ++n) {
      const tthrml_interaction& it = B.interactions[n];
      const int64_t e0 = it.row_ptr[i], e1 = it.row_ptr[i + 1];
      const int n_mult = it.n_sources - it.n_categorical;
      const int64_t cat_prod = it.w_inner / q;
      float contrib[TTHRML_MAX_CATEGORIES];
      for (int k = 0; k < q; ++k) contrib[k] = 0.0f;
      bool first = true;
      for (int64_t e = e0; e < e1; ++e) {
        int64_t sel = 0;
        if (it.n_categorical) sel = cat_select(it, state, C, chain, e);
        const float scale = n_mult ? source_scale(it, state, C, chain, e) : 1.0f;
        for (int k = 0; k < q; ++k) {
          const float w = sel < 0 ? 0.0f : it.weights[e * it.w_inner + k * cat_prod + sel];
          const float term = n_mult ? __fmul_rn(w, scale) : w;
          contrib[k] = first ? term : __fadd_rn(contrib[k], term);
        }
        first = false;
      }
      for (int k = 0; k < q; ++k) theta[k] = seen ? __fadd_rn(theta[k], contrib[k]) : contrib[k];
      seen = true;
    }
    int best = 0;
    if (VARIATES) {
      // argmax(theta + g), first maximum wins (jnp.argmax; tt_thrml/compiler.py:343-344)
      float best_v = 0.0f;
      for (int k = 0; k < q; ++k) {
        const float v = __fadd_rn(theta[k], B.variates[((vsweep * B.n_nodes + i) * q + k) * C + chain]);
        if (k == 0 || v > best_v) {
          best_v = v;
          best = k;
        }
      }
    } else {
      // one uniform per update: counter (chain / 4, row, sweep), word chain % 4
      const u32x4 r = philox4x32_10(u32x4{(uint32_t)(gchain >> 2), (uint32_t)row, sweep, kSaltCat}, k0, k1);
      best = categorical_icdf(theta, q, uniform_open(word_of(r, (int)(gchain & 3))));
    }
    store_value(out, out_idx, (float)best);
  } else {
    bool any_lin, any_prec;
    const float lin = scalar_field(B, 0, state, C, chain, i, &any_lin);
    float prec = scalar_field(B, 1, state, C, chain, i, &any_prec);
    if (!any_prec) prec = 1.0f;
    const float linear = any_lin ? lin : 0.0f;
    // tt_thrml/compiler.py:362-365
    const float inv = 1.0f / __fadd_rn(prec, 1e-6f);
    const float mean = __fmul_rn(linear, inv);
    const float sd = sqrtf(inv);
    float xi;
    if (VARIATES) {
      xi = B.variates[(vsweep * B.n_nodes + i) * C + chain];
    } else {
      const u32x4 r = philox4x32_10(u32x4{(uint32_t)gchain, (uint32_t)row, sweep, kSaltGauss}, k0, k1);
      // Box-Muller on two open uniforms.
      const float u1 = uniform_open(r.x), u2 = uniform_open(r.y);
      xi = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    }
    store_value(out, out_idx, __fadd_rn(mean, __fmul_rn(sd, xi)));
  }
}

template <typename T>
__global__ void __launch_bounds__(256) k_group_commit(tthrml_group g) {
  const int64_t C = g.n_chains;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (tid >= g.group_rows * C) return;
  const int64_t lrow = tid / C;
  const int64_t chain = tid - lrow * C;
  int b = 0;
  int64_t base = 0;
  while (b + 1 < g.n_blocks && lrow >= base + g.blocks[b].n_nodes) {
    base += g.blocks[b].n_nodes;
    ++b;
  }
  const int64_t row = g.blocks[b].row_start + (lrow - base);
  ((T*)g.state)[row * C + chain] = ((const T*)g.scratch)[tid];
}

template <typename T>
int launch_group(const tthrml_group& g, cudaStream_t s) {
  const int64_t total = g.group_rows * g.n_chains;
  if (total == 0) return TTHRML_OK;
  const int threads = 256;
  const int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) {
    set_error("tthrml_group_step: group too large (%lld threads)", (long long)total);
    return TTHRML_ERR_ARG;
  }
  if (g.use_variates)
    k_group_generic<T, true><<<(unsigned)blocks, threads, 0, s>>>(g);
  else
    k_group_generic<T, false><<<(unsigned)blocks, threads, 0, s>>>(g);
  int rc = launch_status("k_group_generic launch");
  if (rc) return rc;
  if (!g.in_place) {
    k_group_commit<T><<<(unsigned)blocks, threads, 0, s>>>(g);
    rc = launch_status("k_group_commit launch");
  }
  return rc;
}

}  // namespace
}  // namespace tthrml

extern "C" int tthrml_group_step(const tthrml_group* g, void* stream) {
  using namespace tthrml;
  if (!g || !g->blocks || !g->state || g->n_blocks <= 0 || g->n_chains <= 0 || g->group_rows < 0) {
    set_error("tthrml_group_step: invalid group descriptor");
    return TTHRML_ERR_ARG;
  }
  if (!g->in_place && !g->scratch) {
    set_error("tthrml_group_step: scratch is required when in_place == 0");
    return TTHRML_ERR_ARG;
  }
  if (g->chain_offset % 4) {
    set_error("tthrml_group_step: chain_offset must be a multiple of 4");
    return TTHRML_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  if (g->state_dtype == TTHRML_STATE_F32) return launch_group<float>(*g, s);
  if (g->state_dtype == TTHRML_STATE_I8) return launch_group<int8_t>(*g, s);
  set_error("tthrml_group_step: unknown state dtype %d", g->state_dtype);
  return TTHRML_ERR_ARG;
}

// ---------------------------------------------------------------------------
// Allocation-free group step.
//
// tthrml_group_step needs a caller-provided scratch buffer whenever a group
// reads its own rows: every block samples from the pre-group state, so new
// values are staged and committed afterwards.  Some hosts cannot hand one over:
// a plugin or FFI host that gives the library only the buffers it owns and has
// no device allocator to lend, or a control loop that must not call cudaMalloc
// (which can synchronise the whole device) once it is running.  For them the
// staging area is this library's own file-scope device array.  With lazy module
// loading (the CUDA 12 default) a device reserves it when this file's kernels
// are first used there, and keeps it until the process exits.  The array's
// device address belongs to the CUDA context that loaded the module: it is
// looked up again on every call made outside stream capture (so a new context,
// e.g. after cudaDeviceReset, gets its own address) and cached per context for
// calls made while the stream is being captured.
// ---------------------------------------------------------------------------
#include <mutex>

namespace tthrml {
namespace {

__device__ __align__(256) unsigned char g_static_scratch[TTHRML_STATIC_SCRATCH_BYTES];

constexpr int kMaxScratchContexts = 64;
std::mutex g_static_scratch_mutex;
struct ScratchAddr {
  void* ctx;
  void* addr;
};
ScratchAddr g_static_scratch_addr[kMaxScratchContexts];  // device address per CUDA context
int g_static_scratch_n = 0;

typedef int (*cu_ctx_get_current_fn)(void**);

// Current CUDA context handle (driver API through the runtime's entry-point
// query, so the library needs no link against libcuda).
int current_context(void** ctx) {
  static cu_ctx_get_current_fn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    const cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p) {
      set_error("tthrml_group_step_static_scratch: cuCtxGetCurrent is unavailable (%s)", cudaGetErrorString(e));
      return TTHRML_ERR_CUDA;
    }
    fn = (cu_ctx_get_current_fn)p;
  }
  *ctx = nullptr;
  const int r = fn(ctx);
  if (r != 0 || !*ctx) {
    set_error("tthrml_group_step_static_scratch: no current CUDA context (driver status %d)", r);
    return TTHRML_ERR_CUDA;
  }
  return TTHRML_OK;
}

// Device address of g_static_scratch in the current context.  Host code only
// sees a host-side stand-in under the array's name, so the address must come
// from cudaGetSymbolAddress with that context current.
int static_scratch_address(cudaStream_t stream, void** out) {
  // a runtime call first: it makes the device's primary context current when no context is
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(stream, &cap);
  if (e != cudaSuccess) return cuda_status(e, "tthrml_group_step_static_scratch: cudaStreamIsCapturing");
  void* ctx = nullptr;
  const int rc = current_context(&ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  int slot = -1;
  for (int i = 0; i < g_static_scratch_n; ++i)
    if (g_static_scratch_addr[i].ctx == ctx) slot = i;
  if (cap == cudaStreamCaptureStatusNone || slot < 0) {
    if (cap != cudaStreamCaptureStatusNone) {
      set_error("tthrml_group_step_static_scratch: the first call in a CUDA context must come before stream capture");
      return TTHRML_ERR_ARG;
    }
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_status(e, "tthrml_group_step_static_scratch: cudaGetSymbolAddress");
    if (slot < 0) {
      if (g_static_scratch_n == kMaxScratchContexts) {  // table full: forget the oldest context
        for (int i = 1; i < kMaxScratchContexts; ++i) g_static_scratch_addr[i - 1] = g_static_scratch_addr[i];
        --g_static_scratch_n;
      }
      slot = g_static_scratch_n++;
      g_static_scratch_addr[slot].ctx = ctx;
    }
    g_static_scratch_addr[slot].addr = p;
  }
  *out = g_static_scratch_addr[slot].addr;
  return TTHRML_OK;
}

}  // namespace
}  // namespace tthrml

extern "C" int tthrml_group_step_static_scratch(const tthrml_group* g, void* stream) {
  using namespace tthrml;
  if (!g || !g->blocks || !g->state || g->n_blocks <= 0 || g->n_chains <= 0 || g->group_rows < 0) {
    set_error("tthrml_group_step_static_scratch: invalid group descriptor");
    return TTHRML_ERR_ARG;
  }
  if (g->chain_offset % 4) {
    set_error("tthrml_group_step_static_scratch: chain_offset must be a multiple of 4");
    return TTHRML_ERR_ARG;
  }
  int64_t elem = 0;
  if (g->state_dtype == TTHRML_STATE_F32) elem = 4;
  if (g->state_dtype == TTHRML_STATE_I8) elem = 1;
  if (!elem) {
    set_error("tthrml_group_step_static_scratch: unknown state dtype %d", g->state_dtype);
    return TTHRML_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  if (g->in_place) return elem == 4 ? launch_group<float>(*g, s) : launch_group<int8_t>(*g, s);  // no staging
  // rows that fit, tested before any product is formed (no signed overflow)
  const int64_t max_rows = (int64_t)TTHRML_STATIC_SCRATCH_BYTES / elem / g->n_chains;
  if (g->group_rows > max_rows) {
    set_error("tthrml_group_step_static_scratch: the group needs %lld rows x %lld chains x %lld B of scratch but "
              "the static scratch holds %lld bytes (%lld rows at this chain count); use tthrml_group_step with a "
              "caller buffer",
              (long long)g->group_rows, (long long)g->n_chains, (long long)elem,
              (long long)TTHRML_STATIC_SCRATCH_BYTES, (long long)max_rows);
    return TTHRML_ERR_ARG;
  }
  void* scratch = nullptr;
  const int rc = static_scratch_address(s, &scratch);
  if (rc) return rc;
  tthrml_group local = *g;
  local.scratch = scratch;
  return elem == 4 ? launch_group<float>(local, s) : launch_group<int8_t>(local, s);
}
