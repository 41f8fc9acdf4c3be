// Shared helpers for the card_playing_gym_b200 native library (sm_100a only).
#pragma once

#include <utility>

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "cg_b200.h"

namespace cg {

// ---- error reporting (capi.cu) ------------------------------------------------
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);

#define CG_REQUIRE(cond, ...)                                  \
  do {                                                         \
    if (!(cond)) return ::cg::set_error(CG_ERR_ARGUMENT, __VA_ARGS__); \
  } while (0)

// Device-side fault word: kernels that give up a bounded wait record where.
// cg_fault_status() reads and clears it.
extern __device__ int g_fault;

__device__ __forceinline__ void raise_fault(int code) { atomicCAS(&g_fault, 0, code); }

// Programmatic dependent launch. A kernel started by launch_pdl may begin while the kernel
// before it in the stream is still running: it may set up (barriers, tensor memory, copies
// of constant weights) but must call pdl_wait() before it reads or writes anything an earlier
// kernel of the stream touches. pdl_trigger(), issued after the wait, lets the next kernel of
// the stream start its own set-up early; so at most two kernels ever overlap.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KernelArgs, typename... Args>
int launch_pdl(const char* what, void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem,
               cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
  if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(err));
  return check_launch(what);
}

// ---- element access by runtime dtype --------------------------------------------
__device__ __forceinline__ float load_as_float(const void* base, int64_t index, int dtype) {
  if (dtype == CG_F32) return static_cast<const float*>(base)[index];
  if (dtype == CG_F16) return __half2float(static_cast<const __half*>(base)[index]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[index]);
}

__device__ __forceinline__ void store_from_float(void* base, int64_t index, int dtype, float value) {
  if (dtype == CG_F32) {
    static_cast<float*>(base)[index] = value;
  } else if (dtype == CG_F16) {
    static_cast<__half*>(base)[index] = __float2half_rn(value);
  } else {
    static_cast<__nv_bfloat16*>(base)[index] = __float2bfloat16_rn(value);
  }
}

__device__ __forceinline__ float round_bf16(float value) {
  return __bfloat162float(__float2bfloat16_rn(value));
}

inline int dtype_size(int dtype) { return dtype == CG_F32 ? 4 : 2; }
inline bool valid_dtype(int dtype) { return dtype == CG_F32 || dtype == CG_F16 || dtype == CG_BF16; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Exact (erf) GELU, as nn.GELU() computes it.
__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

inline int sm_count() {
  static int count = 0;
  if (!count) {
    int device = 0;
    cudaGetDevice(&device);
    cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
    if (!count) count = 148;
  }
  return count;
}

}  // namespace cg
