// Halo exchange of the row-strip lattice decomposition over NVLink peer
// memory, fused with the half-sweep kernel.
//
// Each rank owns one mailbox (device memory it exports with a CUDA IPC handle)
// laid out [2 parity slots][2 directions: from up, from down][2 colours]
// [D rows][W/2], followed by two uint32 flags (from up, from down).  In the
// last two half-sweeps of an exchange period the half-sweep kernel stores
// every boundary row it computes a second time, straight into the up / down
// neighbour's mailbox slot of the period's parity (tthrml_ising2d_halfsweep_x);
// tthrml_halo_signal then publishes the period number in the neighbours'
// flags (system-scope release), and the neighbour's next period starts with
// tthrml_halo_import, which waits for both flags (acquire, bounded) and copies
// its mailbox into its halo rows.  Two parity slots make a slot free again
// before it is rewritten: a rank writes slot p % 2 in period p only after it
// has seen its neighbours finish period p - 1, i.e. after they imported slot
// p % 2 of period p - 2.  The whole period -- import, half-sweeps, signal --
// runs on one stream without the host and is captured in one CUDA graph.
#include <cstring>

#include "common.cuh"

namespace tthrml {
namespace {

constexpr uint32_t kWaitIters = 1u << 21;  // x 512 ns sleep: ~1 s before a wait gives up

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t period_of(uint32_t sweep, uint32_t per, const tthrml_run_ctl* ctl) {
  return (sweep + (ctl ? ctl->sweep : 0u)) / per + 1u;
}

__global__ void k_halo_signal(uint32_t* up_flag, uint32_t* down_flag, uint32_t per, uint32_t sweep,
                              const tthrml_run_ctl* ctl) {
  __threadfence_system();  // the boundary rows stored by earlier kernels precede the flags
  const uint32_t p = period_of(sweep, per, ctl);
  st_release_sys(up_flag, p);
  st_release_sys(down_flag, p);
}

// grid-stride copy of the mailbox of slot (p - 1) % 2 into the halo rows, after
// both neighbours have published period p - 1; period 1 has nothing to import
__global__ void k_halo_import(int8_t* colour0, int8_t* colour1, int64_t half_w, int64_t rows, int64_t top_row0,
                              int64_t bottom_row0, const int8_t* mailbox, const uint32_t* flags, uint32_t per,
                              uint32_t sweep, const tthrml_run_ctl* ctl, int32_t* error) {
  const uint32_t p = period_of(sweep, per, ctl);
  if (p <= 1u) return;
  __shared__ int ok;
  if (threadIdx.x == 0) {
    uint32_t it = 0;
    while (it < kWaitIters && (ld_acquire_sys(flags) < p - 1u || ld_acquire_sys(flags + 1) < p - 1u)) {
      __nanosleep(512);
      ++it;
    }
    ok = it < kWaitIters;
    if (!ok) atomicExch(error, 1);
  }
  __syncthreads();
  if (!ok) return;
  const int64_t plane = rows * half_w;  // one (slot, direction, colour) block
  const int8_t* slot = mailbox + (int64_t)((p - 1u) & 1u) * 4 * plane;
  const int64_t vecs = plane / 16;
  const int64_t total = 4 * vecs;  // 2 directions x 2 colours
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t blk = v / vecs, off = (v - blk * vecs) * 16;
    const int dir = (int)(blk >> 1), c = (int)(blk & 1);
    const uint4 val = *reinterpret_cast<const uint4*>(slot + blk * plane + off);
    int8_t* dst = (c ? colour1 : colour0) + (dir ? bottom_row0 : top_row0) * half_w + off;
    *reinterpret_cast<uint4*>(dst) = val;
  }
}

}  // namespace
}  // namespace tthrml

extern "C" int tthrml_ipc_malloc(int64_t bytes, void** ptr, void* handle) {
  using namespace tthrml;
  if (bytes <= 0 || !ptr || !handle) {
    set_error("tthrml_ipc_malloc: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, (size_t)bytes);
  if (e != cudaSuccess) return cuda_status(e, "tthrml_ipc_malloc: cudaMalloc");
  e = cudaMemset(*ptr, 0, (size_t)bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle), *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return cuda_status(e, "tthrml_ipc_malloc: cudaIpcGetMemHandle");
  }
  return TTHRML_OK;
}

extern "C" int tthrml_ipc_open(const void* handle, void** ptr) {
  using namespace tthrml;
  if (!handle || !ptr) {
    set_error("tthrml_ipc_open: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

extern "C" int tthrml_ipc_close(void* ptr) {
  return tthrml::cuda_status(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
}

extern "C" int tthrml_free(void* ptr) { return tthrml::cuda_status(cudaFree(ptr), "cudaFree"); }

extern "C" int tthrml_memcpy(void* dst, const void* src, int64_t bytes, void* stream) {
  using namespace tthrml;
  if (bytes < 0 || (bytes && (!dst || !src))) {
    set_error("tthrml_memcpy: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  if (!bytes) return TTHRML_OK;
  return cuda_status(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault, (cudaStream_t)stream),
                     "tthrml_memcpy");
}

extern "C" int tthrml_halo_signal(uint32_t* up_flag, uint32_t* down_flag, uint32_t sweeps_per_period,
                                  uint32_t sweep, const tthrml_run_ctl* ctl, void* stream) {
  using namespace tthrml;
  if (!up_flag || !down_flag || sweeps_per_period == 0) {
    set_error("tthrml_halo_signal: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  k_halo_signal<<<1, 1, 0, (cudaStream_t)stream>>>(up_flag, down_flag, sweeps_per_period, sweep, ctl);
  return launch_status("k_halo_signal launch");
}

extern "C" int tthrml_halo_import(int8_t* colour0, int8_t* colour1, int64_t width, int64_t rows, int64_t top_row0,
                                  int64_t bottom_row0, const int8_t* mailbox, const uint32_t* flags,
                                  uint32_t sweeps_per_period, uint32_t sweep, const tthrml_run_ctl* ctl,
                                  int32_t* error, void* stream) {
  using namespace tthrml;
  if (!colour0 || !colour1 || !mailbox || !flags || !error || width <= 0 || width % 32 || rows <= 0 ||
      sweeps_per_period == 0 || top_row0 < 0 || bottom_row0 < 0 || ((uintptr_t)mailbox % 16) ||
      ((uintptr_t)colour0 % 16) || ((uintptr_t)colour1 % 16)) {
    set_error("tthrml_halo_import: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  const int64_t vecs = 4 * rows * (width / 2) / 16;
  const int threads = 256;
  int64_t blocks = (vecs + threads - 1) / threads;
  if (blocks > 1184) blocks = 1184;
  k_halo_import<<<(int)blocks, threads, 0, (cudaStream_t)stream>>>(colour0, colour1, width / 2, rows, top_row0,
                                                                   bottom_row0, mailbox, flags, sweeps_per_period,
                                                                   sweep, ctl, error);
  return launch_status("k_halo_import launch");
}
