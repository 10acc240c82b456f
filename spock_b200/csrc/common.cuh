// Shared helpers for the spock_b200 CUDA kernels (sm_100a only).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "../../include/spock_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "spock_b200 kernels are written for sm_100a (B200) only"
#endif

namespace spock {

// Launch accounting (spock_kernel_launch_count).
extern std::atomic<uint64_t> g_launches;

// Error record filled by the launchers and read by the C ABI layer.
struct Status {
  int code = SPOCK_OK;
  std::string msg;
  static Status ok() { return Status(); }
  static Status err(int c, std::string m) {
    Status s;
    s.code = c;
    s.msg = std::move(m);
    return s;
  }
};

inline Status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return Status::ok();
  return Status::err(SPOCK_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define SPOCK_LAUNCH_CHECK(what)                                   \
  do {                                                             \
    spock::g_launches.fetch_add(1, std::memory_order_relaxed);     \
    cudaError_t _e = cudaGetLastError();                           \
    if (_e != cudaSuccess) return spock::cuda_status(_e, what);    \
  } while (0)

// ---- programmatic dependent launch -----------------------------------------
// The decode step launches its kernels with programmatic stream serialisation
// (pdl_scope), so a kernel's CTAs start while its predecessor drains. Every
// kernel of the step therefore calls pdl_wait() before it reads what the
// predecessor wrote or writes anything the predecessor may still read, and
// pdl_launch() only after that wait (so each grid starts after everything
// before its predecessor has completed). Outside a PDL launch both return at
// once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host: launches made by this thread while a pdl_scope is alive use PDL.
bool& pdl_enabled();
struct pdl_scope {
  bool prev;
  pdl_scope() : prev(pdl_enabled()) { pdl_enabled() = true; }
  ~pdl_scope() { pdl_enabled() = prev; }
};
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}
// launch_k with thread-block clusters of `cluster` CTAs.
template <typename... KArgs, typename... Args>
cudaError_t launch_k_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, dim3 cluster, size_t smem, cudaStream_t st,
                             Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster.x;
  attr[0].val.clusterDim.y = cluster.y;
  attr[0].val.clusterDim.z = cluster.z;
  cfg.numAttrs = 1;
  if (pdl_enabled()) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  cfg.attrs = attr;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ---- device helpers -------------------------------------------------------

// IEEE arithmetic with contraction disabled, so per-element updates round
// exactly as the reference shaders' separate multiply and add.
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

template <typename T>
__device__ __forceinline__ float load_as_f32(const T* p, int64_t i);
template <>
__device__ __forceinline__ float load_as_f32<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float load_as_f32<__half>(const __half* p, int64_t i) {
  return __half2float(p[i]);
}
template <>
__device__ __forceinline__ float load_as_f32<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

}  // namespace spock
