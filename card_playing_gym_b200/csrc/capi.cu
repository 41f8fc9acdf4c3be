// Error state, version and the device fault word of the C ABI.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace cg {

namespace {
thread_local char g_message[1024] = "";
int64_t g_launches = 0;
}

__device__ int g_fault = 0;

int set_error(int code, const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_message, sizeof(g_message), fmt, args);
  va_end(args);
  return code;
}

int check_launch(const char* what) {
  ++g_launches;
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
  return CG_OK;
}

}  // namespace cg

extern "C" const char* cg_last_error(void) { return cg::g_message; }

extern "C" int cg_version(void) { return 1; }

extern "C" int64_t cg_launch_count(void) { return cg::g_launches; }

extern "C" int cg_fault_status(int* code_out) {
  if (!code_out) return cg::set_error(CG_ERR_ARGUMENT, "cg_fault_status: code_out is NULL");
  cudaError_t err = cudaDeviceSynchronize();
  if (err != cudaSuccess) return cg::set_error(CG_ERR_CUDA, "cg_fault_status: %s", cudaGetErrorString(err));
  int zero = 0;
  err = cudaMemcpyFromSymbol(code_out, cg::g_fault, sizeof(int));
  if (err == cudaSuccess) err = cudaMemcpyToSymbol(cg::g_fault, &zero, sizeof(int));
  if (err != cudaSuccess) return cg::set_error(CG_ERR_CUDA, "cg_fault_status: %s", cudaGetErrorString(err));
  return CG_OK;
}
