// KV pool maintenance: per-row writes and row copies (cardgym/nn/kv_cache.py:84-105, 122-138).
//
// Row and position indices come from the caller's device buffers, so they are checked on the
// device: an index outside the pool is skipped (nothing is read or written through it) and the
// device fault word is set (0x110 for a write, 0x111 for a row copy), which cg_fault_status()
// reports. The reference's torch indexing raises on such an index instead.
#include <mutex>

#include <cuda.h>

#include "common.cuh"

namespace cg {

// k_new/v_new [B, KVH, T, D] -> pool[rows[b], kvh, positions[b, t], :]
__global__ void kv_write_step_kernel(void* k_layer, void* v_layer, int kv_dtype, int64_t capacity, int kv_heads,
                                     int max_len, int head_dim, const int64_t* rows, const int64_t* positions,
                                     int64_t batch, int steps, const void* k_new, const void* v_new, int src_dtype) {
  const int64_t total = batch * kv_heads * steps * head_dim;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int d = static_cast<int>(i % head_dim);
    const int t = static_cast<int>((i / head_dim) % steps);
    const int kvh = static_cast<int>((i / (static_cast<int64_t>(head_dim) * steps)) % kv_heads);
    const int64_t b = i / (static_cast<int64_t>(head_dim) * steps * kv_heads);
    const int64_t row = rows ? rows[b] : b;
    const int64_t pos = positions[b * steps + t];
    if (row < 0 || row >= capacity || pos < 0 || pos >= max_len) {
      if (d == 0) raise_fault(0x110);
      continue;
    }
    const int64_t dst = ((row * kv_heads + kvh) * max_len + pos) * head_dim + d;
    store_from_float(k_layer, dst, kv_dtype, load_as_float(k_new, i, src_dtype));
    store_from_float(v_layer, dst, kv_dtype, load_as_float(v_new, i, src_dtype));
  }
}

// Gather (to_stage=1: from sources) or scatter (to_stage=0: to targets) `count` rows of every
// layer, first `length` positions. The stage holds [count, n_layers, 2, KVH, length, D] in
// 16-byte words when the row width allows. A pair whose source or target lies outside
// [0, capacity) is skipped by both passes, so nothing stale is ever scattered.
__global__ void kv_stage_kernel(unsigned char* k_pool, unsigned char* v_pool, unsigned char* stage, int n_layers,
                                int64_t capacity, int kv_heads, int max_len, int64_t row_bytes_pos,
                                const int64_t* sources, const int64_t* targets, int64_t count, int length,
                                int to_stage) {
  // One "segment" = one (row, layer, k|v, head): `length * row_bytes_pos` contiguous bytes.
  const int64_t seg_bytes = static_cast<int64_t>(length) * row_bytes_pos;
  const int64_t segs = count * n_layers * 2 * kv_heads;
  const bool vec = (seg_bytes % 16 == 0) && (row_bytes_pos * max_len % 16 == 0);
  const int64_t unit = vec ? 16 : 1;
  const int64_t per_seg = seg_bytes / unit;
  const int64_t total = segs * per_seg;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t seg = i / per_seg, w = i % per_seg;
    const int kvh = static_cast<int>(seg % kv_heads);
    const int which = static_cast<int>((seg / kv_heads) % 2);
    const int layer = static_cast<int>((seg / (2 * kv_heads)) % n_layers);
    const int64_t r = seg / (2 * kv_heads * static_cast<int64_t>(n_layers));
    const int64_t source = sources[r], target = targets[r];
    if (source < 0 || source >= capacity || target < 0 || target >= capacity) {
      if (to_stage && w == 0) raise_fault(0x111);
      continue;
    }
    const int64_t row = to_stage ? source : target;
    unsigned char* pool = which ? v_pool : k_pool;
    const int64_t pool_off = (((static_cast<int64_t>(layer) * capacity + row) * kv_heads + kvh) * max_len) * row_bytes_pos;
    unsigned char* a = pool + pool_off + w * unit;
    unsigned char* s = stage + seg * seg_bytes + w * unit;
    if (vec) {
      if (to_stage) *reinterpret_cast<uint4*>(s) = *reinterpret_cast<const uint4*>(a);
      else *reinterpret_cast<uint4*>(a) = *reinterpret_cast<const uint4*>(s);
    } else {
      if (to_stage) *s = *a;
      else *a = *s;
    }
  }
}

}  // namespace cg

extern "C" int cg_kv_write_step(void* k_layer, void* v_layer, int kv_dtype, int64_t capacity, int kv_heads, int max_len,
                                int head_dim, const int64_t* rows, const int64_t* positions, int64_t batch, int steps,
                                const void* k_new, const void* v_new, int src_dtype, void* stream) {
  using namespace cg;
  CG_REQUIRE(valid_dtype(kv_dtype) && valid_dtype(src_dtype), "cg_kv_write_step: bad dtype");
  CG_REQUIRE(batch >= 0 && steps > 0 && kv_heads > 0 && head_dim > 0 && max_len > 0, "cg_kv_write_step: bad shape");
  if (batch == 0) return CG_OK;
  CG_REQUIRE(k_layer && v_layer && positions && k_new && v_new, "cg_kv_write_step: NULL pointer");
  CG_REQUIRE(capacity > 0, "cg_kv_write_step: bad capacity");
  const int64_t total = batch * kv_heads * steps * head_dim;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 65535) blocks = 65535;
  kv_write_step_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      k_layer, v_layer, kv_dtype, capacity, kv_heads, max_len, head_dim, rows, positions, batch, steps, k_new, v_new,
      src_dtype);
  return check_launch("kv_write_step_kernel");
}

extern "C" int64_t cg_kv_copy_rows_workspace_bytes(int n_layers, int kv_heads, int max_len, int head_dim, int kv_dtype,
                                                   int64_t count) {
  return count * n_layers * 2LL * kv_heads * max_len * head_dim * cg::dtype_size(kv_dtype);
}

extern "C" int cg_kv_copy_rows(void* k_pool, void* v_pool, int kv_dtype, int n_layers, int64_t capacity, int kv_heads,
                               int max_len, int head_dim, const int64_t* sources, const int64_t* targets, int64_t count,
                               int length, void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace cg;
  CG_REQUIRE(valid_dtype(kv_dtype), "cg_kv_copy_rows: bad dtype");
  CG_REQUIRE(count >= 0 && length >= 0 && length <= max_len, "cg_kv_copy_rows: bad count/length");
  if (count == 0 || length == 0) return CG_OK;
  CG_REQUIRE(k_pool && v_pool && sources && targets && workspace, "cg_kv_copy_rows: NULL pointer");
  const int64_t row_bytes_pos = static_cast<int64_t>(head_dim) * dtype_size(kv_dtype);
  const int64_t need = count * n_layers * 2LL * kv_heads * length * row_bytes_pos;
  if (workspace_bytes < need)
    return set_error(CG_ERR_WORKSPACE, "cg_kv_copy_rows: workspace %lld < %lld bytes", (long long)workspace_bytes,
                     (long long)need);
  CG_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 15) == 0, "cg_kv_copy_rows: workspace must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int blocks = sm_count() * 8;
  kv_stage_kernel<<<blocks, 256, 0, s>>>(static_cast<unsigned char*>(k_pool), static_cast<unsigned char*>(v_pool),
                                         static_cast<unsigned char*>(workspace), n_layers, capacity, kv_heads, max_len,
                                         row_bytes_pos, sources, targets, count, length, 1);
  int rc = check_launch("kv_stage_kernel(gather)");
  if (rc) return rc;
  kv_stage_kernel<<<blocks, 256, 0, s>>>(static_cast<unsigned char*>(k_pool), static_cast<unsigned char*>(v_pool),
                                         static_cast<unsigned char*>(workspace), n_layers, capacity, kv_heads, max_len,
                                         row_bytes_pos, sources, targets, count, length, 0);
  return check_launch("kv_stage_kernel(scatter)");
}

// ---------------------------------------------------------------------------------------
// Row copies without any allocation.
//
// Some callers cannot allocate device memory around a copy: a collector loop that steps
// games on the host while the device works cannot afford cudaMalloc (it synchronizes the
// device), and a host embedding this library through its C ABI may have no allocator of
// its own (the device memory belongs to another framework's pool). For them the staging
// buffer lives in this file-scope array, which every GPU that loads the library holds
// until the process exits.
// ---------------------------------------------------------------------------------------
namespace {
constexpr int64_t kNoAllocScratchBytes = 16LL << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_copy_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mutex;

// The address of g_copy_scratch belongs to one CUDA context: after cudaDeviceReset, or under
// a context other than the device's primary one, an address taken earlier is dead or foreign.
// So it is remembered per (device, current context) and looked up again on every call made
// outside stream capture; a call inside a capture reuses the address its context recorded.
struct ScratchEntry {
  int device;
  CUcontext context;
  unsigned char* address;
};
ScratchEntry g_scratch_entries[64];
int g_scratch_count = 0;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CUcontext current_context() {
  static CtxGetCurrentFn fn = [] {
    void* entry = nullptr;
    cudaDriverEntryPointQueryResult found = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &entry, cudaEnableDefault, &found) != cudaSuccess ||
        found != cudaDriverEntryPointSuccess)
      entry = nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(entry);
  }();
  CUcontext context = nullptr;
  if (fn) fn(&context);
  return context;
}

// Device address of g_copy_scratch for the current device and context. The host-side name
// is only a stand-in for the symbol, so the address comes from cudaGetSymbolAddress with that
// device current; the first call on a device (or after a reset) must come before any capture.
int scratch_address(cudaStream_t stream, unsigned char** out) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return cg::set_error(CG_ERR_CUDA, "cg_kv_copy_rows_noalloc: %s", cudaGetErrorString(err));
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  err = cudaStreamIsCapturing(stream, &capture);
  if (err != cudaSuccess) return cg::set_error(CG_ERR_CUDA, "cg_kv_copy_rows_noalloc: %s", cudaGetErrorString(err));
  const CUcontext context = current_context();
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchEntry* entry = nullptr;
  for (int i = 0; i < g_scratch_count; ++i)
    if (g_scratch_entries[i].device == device && g_scratch_entries[i].context == context) entry = &g_scratch_entries[i];
  if (entry && capture != cudaStreamCaptureStatusNone) {
    *out = entry->address;
    return CG_OK;
  }
  if (!entry && capture != cudaStreamCaptureStatusNone)
    return cg::set_error(CG_ERR_ARGUMENT,
                         "cg_kv_copy_rows_noalloc: the first call on device %d (or after a device reset) must come "
                         "before stream capture",
                         device);
  void* ptr = nullptr;
  err = cudaGetSymbolAddress(&ptr, g_copy_scratch);
  if (err != cudaSuccess)
    return cg::set_error(CG_ERR_CUDA, "cg_kv_copy_rows_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(err));
  if (!entry) {
    if (g_scratch_count == 64) g_scratch_count = 0;  // forget the oldest contexts rather than fail
    entry = &g_scratch_entries[g_scratch_count++];
    entry->device = device;
    entry->context = context;
  }
  entry->address = static_cast<unsigned char*>(ptr);
  *out = entry->address;
  return CG_OK;
}
}  // namespace

extern "C" int64_t cg_kv_copy_rows_noalloc_max_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int cg_kv_copy_rows_noalloc(void* k_pool, void* v_pool, int kv_dtype, int n_layers, int64_t capacity,
                                       int kv_heads, int max_len, int head_dim, const int64_t* sources,
                                       const int64_t* targets, int64_t count, int length, void* stream) {
  using namespace cg;
  CG_REQUIRE(valid_dtype(kv_dtype), "cg_kv_copy_rows_noalloc: bad dtype");
  CG_REQUIRE(count >= 0 && length >= 0 && length <= max_len, "cg_kv_copy_rows_noalloc: bad count/length");
  if (count == 0 || length == 0) return CG_OK;
  CG_REQUIRE(k_pool && v_pool && sources && targets, "cg_kv_copy_rows_noalloc: NULL pointer");
  const int64_t row_bytes_pos = static_cast<int64_t>(head_dim) * dtype_size(kv_dtype);
  const int64_t need = count * n_layers * 2LL * kv_heads * length * row_bytes_pos;
  if (need > kNoAllocScratchBytes)
    return set_error(CG_ERR_ARGUMENT,
                     "cg_kv_copy_rows_noalloc: %lld rows x %d positions need %lld staging bytes, above its fixed "
                     "%lld-byte buffer; split the copy into smaller calls",
                     (long long)count, length, (long long)need, (long long)kNoAllocScratchBytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned char* scratch = nullptr;
  int rc = scratch_address(s, &scratch);
  if (rc) return rc;
  // The gather writes every staged byte before the scatter reads it: nothing needs clearing.
  const int blocks = sm_count() * 8;
  kv_stage_kernel<<<blocks, 256, 0, s>>>(static_cast<unsigned char*>(k_pool), static_cast<unsigned char*>(v_pool),
                                         scratch, n_layers, capacity, kv_heads, max_len, row_bytes_pos, sources,
                                         targets, count, length, 1);
  if ((rc = check_launch("kv_stage_kernel(gather, no-alloc)"))) return rc;
  kv_stage_kernel<<<blocks, 256, 0, s>>>(static_cast<unsigned char*>(k_pool), static_cast<unsigned char*>(v_pool),
                                         scratch, n_layers, capacity, kv_heads, max_len, row_bytes_pos, sources,
                                         targets, count, length, 0);
  return check_launch("kv_stage_kernel(scatter, no-alloc)");
}
