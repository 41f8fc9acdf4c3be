// Ragged GQA decode attention straight from the KV pool.
//
// Reference: cardgym/nn/cuda_decode.py:46-151 (kernel + op) and the PyTorch path it
// short-cuts, cardgym/nn/trunk.py:203-256. Row b appends T tokens at its own length;
// query t of row b sees keys < min(lengths[b] + t, span). The merged query axis of
// a KV head is g * T + t (trunk.py:243-254).
//
// Two kernels:
//  * attn_tc: fp16/bf16 caches, head_dim a multiple of 8, G*T <= 16. One warp per
//    (row, KV head) unit, persistent over units. Each warp streams its unit's keys in
//    chunks of 64 through a two-stage shared-memory ring filled by bulk async copies
//    (cp.async.bulk, completion on an mbarrier), computes Q K^T and P V with
//    mma.sync m16n8k16/k8 (fp32 accumulation) and keeps an online softmax in fp32.
//  * attn_simt: any cache dtype and shape; one warp per (row, query head, step),
//    fp32 arithmetic. Used for fp32 caches (the strict-parity mode) and shapes the
//    tensor-core kernel does not take.
#include "trunk.h"

namespace cg {



// ------------------------------------------------------------------------------------
// SIMT kernel: warp per (b, head, t); lanes stride the keys; online softmax.
// ------------------------------------------------------------------------------------
constexpr int kSimtMaxDim = 128;

__global__ void __launch_bounds__(128) attn_simt_kernel(AttnParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t total = p.batch * p.heads * p.steps;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int D = p.head_dim;
  __shared__ float q_s[4][kSimtMaxDim];
  float* qv = q_s[threadIdx.x >> 5];
  for (int64_t item = warp; item < total; item += warps) {
    const int t = static_cast<int>(item % p.steps);
    const int h = static_cast<int>((item / p.steps) % p.heads);
    const int64_t b = item / (static_cast<int64_t>(p.steps) * p.heads);
    const int kvh = h / p.group;
    const int64_t row = p.rows ? p.rows[b] : b;
    const int64_t limit64 = p.lengths[b] + t;
    const int limit = static_cast<int>(limit64 < p.span ? limit64 : p.span);
    const int64_t qoff = b * p.q_sb + h * p.q_sh + t * p.q_st;
    __syncwarp();
    for (int d = lane; d < D; d += 32) qv[d] = load_as_float(p.q, qoff + d, p.q_dtype);
    __syncwarp();
    const int64_t base = row * p.kv_row + kvh * p.kv_head;
    float m = -INFINITY, l = 0.f;
    float acc[kSimtMaxDim / 32];
#pragma unroll
    for (int i = 0; i < kSimtMaxDim / 32; ++i) acc[i] = 0.f;
    for (int c0 = 0; c0 < limit; c0 += 32) {
      const int key = c0 + lane;
      float s = -INFINITY;
      if (key < limit) {
        const int64_t off = base + key * p.kv_pos;
        float dot = 0.f;
        for (int d = 0; d < D; ++d) dot = fmaf(qv[d], load_as_float(p.k, off + d, p.kv_dtype), dot);
        s = dot * p.scale;
      }
      const float m_new = fmaxf(m, warp_max(s));
      const float alpha = expf(m - m_new);
      const float pk = key < limit ? expf(s - m_new) : 0.f;
      l = l * alpha + warp_sum(pk);
      const int n = min(32, limit - c0);
#pragma unroll
      for (int i = 0; i < kSimtMaxDim / 32; ++i) acc[i] *= alpha;
      for (int j = 0; j < n; ++j) {
        const float pj = __shfl_sync(0xffffffffu, pk, j);
        const int64_t off = base + (c0 + j) * p.kv_pos;
#pragma unroll
        for (int i = 0; i < kSimtMaxDim / 32; ++i) {
          const int d = lane + 32 * i;
          if (d < D) acc[i] = fmaf(pj, load_as_float(p.v, off + d, p.kv_dtype), acc[i]);
        }
      }
      m = m_new;
    }
    const float inv = limit > 0 ? 1.f / l : 0.f;
    const int64_t ooff = b * p.o_sb + h * p.o_sh + t * p.o_st;
#pragma unroll
    for (int i = 0; i < kSimtMaxDim / 32; ++i) {
      const int d = lane + 32 * i;
      if (d >= D) continue;
      if (p.out_blocked)
        store_from_float(p.out, blocked_offset(b * p.steps + t, h * D + d, p.blocked_width), p.out_dtype, acc[i] * inv);
      else
        store_from_float(p.out, ooff + d, p.out_dtype, acc[i] * inv);
    }
  }
}

// ------------------------------------------------------------------------------------
// Tensor-core kernel.
// ------------------------------------------------------------------------------------
constexpr int kChunk = 64;   // keys per staged chunk
constexpr int kStages = 2;   // chunks in flight per warp
constexpr int kTcWarps = 4;  // warps per CTA
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // bounded mbarrier wait: 1 s

__device__ __forceinline__ uint32_t smem_addr(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

__device__ __forceinline__ uint64_t global_timer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Returns false (and records a fault) if the phase does not complete within the limit.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int fault_code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer() - start > kWaitLimitNs) {
      raise_fault(fault_code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// The KV stream is read once per layer: evict it from L2 first so that weights stay resident.
__device__ __forceinline__ void bulk_copy_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                     uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <typename T>
struct MmaOps;

template <>
struct MmaOps<__half> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ void k16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ void k8(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(b0));
  }
};

template <>
struct MmaOps<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ void k16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ void k8(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(b0));
  }
};

__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename KV, int D>
struct TcShape {
  static constexpr int kTiles = D / 16;          // full k16 blocks of Q K^T
  static constexpr bool kTail = (D % 16) != 0;   // one trailing k8 block
  static constexpr int kDTiles = D / 8;          // n8 tiles of the output
  static constexpr int kStageElems = kChunk * D; // per K or V
  static constexpr int kWarpBytes = kStages * 2 * kStageElems * static_cast<int>(sizeof(KV));
};

// Rows with no visible key get a zero output.
__device__ void zero_unit(const AttnParams& p, int64_t b, int kvh, int M, int lane) {
  const int D = p.head_dim;
  for (int i = lane; i < M * D; i += 32) {
    const int m = i / D, d = i % D;
    const int h = kvh * p.group + m / p.steps, t = m % p.steps;
    const int64_t off = p.out_blocked ? blocked_offset(b * p.steps + t, h * D + d, p.blocked_width)
                                      : b * p.o_sb + h * p.o_sh + t * p.o_st + d;
    store_from_float(p.out, off, p.out_dtype, 0.f);
  }
}

template <typename KV, int D>
__global__ void __launch_bounds__(kTcWarps * 32) attn_tc_kernel(AttnParams p) {
  using Shape = TcShape<KV, D>;
  using Ops = MmaOps<KV>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bars[kTcWarps][kStages];

  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int gid = lane >> 2, tid4 = lane & 3;
  KV* stage_base = reinterpret_cast<KV*>(smem_raw + wib * Shape::kWarpBytes);
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[wib][s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();

  const int64_t units = p.batch * p.kv_heads;
  const int64_t warp0 = static_cast<int64_t>(blockIdx.x) * kTcWarps + wib;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kTcWarps;
  const int M = p.group * p.steps;
  const float scale_log2 = p.scale * 1.4426950408889634f;

  // Visible-key count of the unit's last query (the chunk loop bound).
  auto unit_keys = [&](int64_t unit) -> int {
    const int64_t b = unit / p.kv_heads;
    const int64_t last = p.lengths[b] + p.steps - 1;
    return static_cast<int>(last < p.span ? last : p.span);
  };
  auto issue = [&](int64_t unit, int chunk, int keys, int stage) {
    // Every lane fences its own earlier generic accesses to the stage before the
    // asynchronous copy overwrites it; lane 0 then issues both copies.
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      const int64_t b = unit / p.kv_heads;
      const int kvh = static_cast<int>(unit % p.kv_heads);
      const int64_t row = p.rows ? p.rows[b] : b;
      const int first = chunk * kChunk;
      const int n = min(kChunk, keys - first);
      const uint32_t bytes = static_cast<uint32_t>(n * D * sizeof(KV));
      const int64_t off = row * p.kv_row + kvh * p.kv_head + static_cast<int64_t>(first) * p.kv_pos;
      KV* ks = stage_base + stage * 2 * Shape::kStageElems;
      mbar_expect_tx(&bars[wib][stage], 2 * bytes);
      const uint64_t policy = evict_first_policy();
      bulk_copy_g2s_stream(ks, static_cast<const KV*>(p.k) + off, bytes, &bars[wib][stage], policy);
      bulk_copy_g2s_stream(ks + Shape::kStageElems, static_cast<const KV*>(p.v) + off, bytes, &bars[wib][stage], policy);
    }
  };

  // Find this warp's first unit with at least one key.
  int64_t unit = warp0;
  int keys = 0;
  while (unit < units && (keys = unit_keys(unit)) <= 0) {
    // No visible key: the output is defined as zero.
    const int64_t b = unit / p.kv_heads;
    const int kvh = static_cast<int>(unit % p.kv_heads);
    zero_unit(p, b, kvh, M, lane);
    unit += stride;
  }
  if (unit >= units) return;
  int chunk = 0, stage = 0;
  uint32_t phase[kStages] = {0, 0};
  issue(unit, 0, keys, 0);

  uint32_t qa[Shape::kTiles > 0 ? Shape::kTiles : 1][4];
  uint32_t qt[2];
  float o[Shape::kDTiles][4];
  float mrow[2], lrow[2];
  int limit_r[2];

  while (true) {
    // Next item: the next chunk of this unit, or the first chunk of the next unit with keys.
    int64_t next_unit = unit;
    int next_chunk = chunk + 1, next_keys = keys;
    if (next_chunk * kChunk >= keys) {
      next_chunk = 0;
      next_unit = unit + stride;
      while (next_unit < units && (next_keys = unit_keys(next_unit)) <= 0) {
        const int64_t b = next_unit / p.kv_heads;
        const int kvh = static_cast<int>(next_unit % p.kv_heads);
        zero_unit(p, b, kvh, M, lane);
        next_unit += stride;
      }
    }
    const bool has_next = next_unit < units;
    if (has_next) issue(next_unit, next_chunk, next_keys, stage ^ 1);

    const int64_t b = unit / p.kv_heads;
    const int kvh = static_cast<int>(unit % p.kv_heads);
    if (chunk == 0) {
      // Unit start: Q fragments (rows m >= M are zero), softmax state, limits.
      auto qval = [&](int m, int d) -> float {
        if (m >= M) return 0.f;
        const int h = kvh * p.group + m / p.steps, t = m % p.steps;
        return load_as_float(p.q, b * p.q_sb + h * p.q_sh + t * p.q_st + d, p.q_dtype);
      };
#pragma unroll
      for (int kb = 0; kb < Shape::kTiles; ++kb) {
        const int c = kb * 16 + 2 * tid4;
        qa[kb][0] = Ops::pack(qval(gid, c), qval(gid, c + 1));
        qa[kb][1] = Ops::pack(qval(gid + 8, c), qval(gid + 8, c + 1));
        qa[kb][2] = Ops::pack(qval(gid, c + 8), qval(gid, c + 9));
        qa[kb][3] = Ops::pack(qval(gid + 8, c + 8), qval(gid + 8, c + 9));
      }
      if (Shape::kTail) {
        const int c = Shape::kTiles * 16 + 2 * tid4;
        qt[0] = Ops::pack(qval(gid, c), qval(gid, c + 1));
        qt[1] = Ops::pack(qval(gid + 8, c), qval(gid + 8, c + 1));
      }
#pragma unroll
      for (int j = 0; j < Shape::kDTiles; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int m = gid + 8 * r;
        // Padding rows (m >= M) attend to every visible key: finite, never stored.
        const int t = m < M ? m % p.steps : p.steps - 1;
        const int64_t lim = p.lengths[b] + t;
        limit_r[r] = static_cast<int>(lim < p.span ? lim : p.span);
        mrow[r] = -INFINITY;
        lrow[r] = 0.f;
      }
    }

    if (!mbar_wait_bounded(&bars[wib][stage], phase[stage], 0x100 + wib)) return;
    phase[stage] ^= 1u;
    const KV* ks = stage_base + stage * 2 * Shape::kStageElems;
    const KV* vs = ks + Shape::kStageElems;
    const int first = chunk * kChunk;
    const int n = min(kChunk, keys - first);
    if (n < kChunk && (n & 15)) {
      // Zero the V rows the last partial 16-key block would read: stale shared memory
      // times a zero probability must not turn into NaN.
      KV* vz = const_cast<KV*>(vs);
      const int end = min(kChunk, (n + 15) & ~15);
      for (int i = n * D + lane; i < end * D; i += 32) vz[i] = KV(0.f);
      __syncwarp();
    }
    const int nblocks = (n + 15) >> 4;  // 16-key blocks with any valid key

    // S = Q K^T over the chunk, masked; online softmax update.
    float s[kChunk / 8][4];
    float cmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < kChunk / 8; ++j) {
      s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
      if (j < 2 * nblocks) {
        const KV* krow = ks + (j * 8 + gid) * D;
#pragma unroll
        for (int kb = 0; kb < Shape::kTiles; ++kb) {
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(krow + kb * 16 + 2 * tid4);
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(krow + kb * 16 + 8 + 2 * tid4);
          Ops::k16(s[j], qa[kb], b0, b1);
        }
        if (Shape::kTail) {
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(krow + Shape::kTiles * 16 + 2 * tid4);
          Ops::k8(s[j], qt[0], qt[1], b0);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = first + j * 8 + 2 * tid4 + (e & 1);
        const int r = e >> 1;
        const float v = key < limit_r[r] ? s[j][e] * scale_log2 : -INFINITY;
        s[j][e] = v;
        cmax[r] = fmaxf(cmax[r], v);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      cmax[r] = fmaxf(cmax[r], __shfl_xor_sync(0xffffffffu, cmax[r], 1));
      cmax[r] = fmaxf(cmax[r], __shfl_xor_sync(0xffffffffu, cmax[r], 2));
      const float m_new = fmaxf(mrow[r], cmax[r]);
      alpha[r] = m_new == -INFINITY ? 1.f : exp2f(mrow[r] - m_new);
      mrow[r] = m_new;
    }
    float psum[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < kChunk / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const float pe = s[j][e] == -INFINITY ? 0.f : exp2f(s[j][e] - mrow[r]);
        s[j][e] = pe;
        psum[r] += pe;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) lrow[r] = lrow[r] * alpha[r] + psum[r];
#pragma unroll
    for (int j = 0; j < Shape::kDTiles; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }

    // O += P V, 16 keys at a time.
#pragma unroll
    for (int kk = 0; kk < kChunk / 16; ++kk) {
      if (kk < nblocks) {
        uint32_t pa[4];
        pa[0] = Ops::pack(s[2 * kk][0], s[2 * kk][1]);
        pa[1] = Ops::pack(s[2 * kk][2], s[2 * kk][3]);
        pa[2] = Ops::pack(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        pa[3] = Ops::pack(s[2 * kk + 1][2], s[2 * kk + 1][3]);
        const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int dt = 0; dt < Shape::kDTiles; dt += 2) {
          if (dt + 1 < Shape::kDTiles) {
            const int col = (dt + (lane >> 4)) * 8;
            uint32_t r0, r1, r2, r3;
            ldmatrix_x4_trans(r0, r1, r2, r3, smem_addr(vs + key * D + col));
            Ops::k16(o[dt], pa, r0, r1);
            Ops::k16(o[dt + 1], pa, r2, r3);
          } else {
            uint32_t r0, r1;
            ldmatrix_x2_trans(r0, r1, smem_addr(vs + key * D + dt * 8));
            Ops::k16(o[dt], pa, r0, r1);
          }
        }
      }
    }

    if (next_chunk == 0) {
      // Unit done: normalise and store rows m < M.
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int m = gid + 8 * r;
        if (m < M) {
          const float inv = 1.f / lrow[r];
          const int h = kvh * p.group + m / p.steps, t = m % p.steps;
          const int64_t ooff = b * p.o_sb + h * p.o_sh + t * p.o_st;
#pragma unroll
          for (int j = 0; j < Shape::kDTiles; ++j) {
            const int d = j * 8 + 2 * tid4;
            if (p.out_blocked) {
              // even column pair inside one 8-column chunk: one 32-bit store of two bf16
              const int64_t off = blocked_offset(b * p.steps + t, h * D + d, p.blocked_width);
              *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(p.out) + off) =
                  __floats2bfloat162_rn(o[j][2 * r] * inv, o[j][2 * r + 1] * inv);
            } else {
              store_from_float(p.out, ooff + d, p.out_dtype, o[j][2 * r] * inv);
              store_from_float(p.out, ooff + d + 1, p.out_dtype, o[j][2 * r + 1] * inv);
            }
          }
        }
      }
    }
    __syncwarp();
    if (!has_next) break;
    unit = next_unit;
    chunk = next_chunk;
    keys = next_keys;
    stage ^= 1;
  }
}

template <typename KV, int D>
int launch_tc(const AttnParams& p, cudaStream_t stream) {
  using Shape = TcShape<KV, D>;
  const int smem = kTcWarps * Shape::kWarpBytes;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(attn_tc_kernel<KV, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured = true;
  }
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_tc_kernel<KV, D>, kTcWarps * 32, smem);
  if (per_sm < 1) per_sm = 1;
  const int64_t units = p.batch * p.kv_heads;
  int64_t blocks = static_cast<int64_t>(sm_count()) * per_sm;
  const int64_t needed = (units + kTcWarps - 1) / kTcWarps;
  if (blocks > needed) blocks = needed;
  if (blocks < 1) return CG_OK;
  attn_tc_kernel<KV, D><<<static_cast<unsigned>(blocks), kTcWarps * 32, smem, stream>>>(p);
  return check_launch("attn_tc_kernel");
}

template <typename KV>
int dispatch_tc(const AttnParams& p, cudaStream_t stream) {
  switch (p.head_dim) {
    case 16: return launch_tc<KV, 16>(p, stream);
    case 24: return launch_tc<KV, 24>(p, stream);
    case 32: return launch_tc<KV, 32>(p, stream);
    case 40: return launch_tc<KV, 40>(p, stream);
    case 48: return launch_tc<KV, 48>(p, stream);
    case 64: return launch_tc<KV, 64>(p, stream);
    default: return -1;
  }
}

bool tc_eligible(const AttnParams& p) {
  if (p.kv_dtype == CG_F32) return false;
  if (p.group * p.steps > 16) return false;
  const int d = p.head_dim;
  if (!(d == 16 || d == 24 || d == 32 || d == 40 || d == 48 || d == 64)) return false;
  // Bulk copies need 16-byte aligned sources: contiguous key rows, aligned row/head strides.
  if (p.kv_pos != d) return false;
  if ((p.kv_row % 8) || (p.kv_head % 8)) return false;
  if ((reinterpret_cast<uintptr_t>(p.k) & 15) || (reinterpret_cast<uintptr_t>(p.v) & 15)) return false;
  return true;
}

namespace {
struct AttentionProfile {
  bool enabled = false;
  int capacity = 0;
  int count = 0;
  cudaEvent_t* start = nullptr;
  cudaEvent_t* stop = nullptr;
} g_profile;
}  // namespace

int profile_attention(int enable, int capacity) {
  for (int i = 0; i < g_profile.capacity; ++i) {
    cudaEventDestroy(g_profile.start[i]);
    cudaEventDestroy(g_profile.stop[i]);
  }
  delete[] g_profile.start;
  delete[] g_profile.stop;
  g_profile = AttentionProfile{};
  if (!enable) return CG_OK;
  CG_REQUIRE(capacity > 0 && capacity <= (1 << 20), "cg_attention_profiling: capacity 1..2^20");
  g_profile.start = new cudaEvent_t[capacity];
  g_profile.stop = new cudaEvent_t[capacity];
  for (int i = 0; i < capacity; ++i) {
    if (cudaEventCreate(&g_profile.start[i]) != cudaSuccess || cudaEventCreate(&g_profile.stop[i]) != cudaSuccess) {
      g_profile.capacity = i;
      return set_error(CG_ERR_CUDA, "cg_attention_profiling: cudaEventCreate failed");
    }
    g_profile.capacity = i + 1;
  }
  g_profile.enabled = true;
  return CG_OK;
}

int attention_timings(float* ms_out, int max_count) {
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  const int n = g_profile.count < max_count ? g_profile.count : max_count;
  for (int i = 0; i < n; ++i) {
    if (cudaEventElapsedTime(&ms_out[i], g_profile.start[i], g_profile.stop[i]) != cudaSuccess) return -1;
  }
  return n;
}

int run_attention_kernels(const AttnParams& p, cudaStream_t stream);

int run_attention(const AttnParams& p, cudaStream_t stream) {
  if (p.batch == 0) return CG_OK;
  if (p.out_blocked && (p.out_dtype != CG_BF16 || p.blocked_width != p.heads * p.head_dim || p.blocked_width % 8))
    return set_error(CG_ERR_ARGUMENT, "blocked attention output must be bf16 with width heads*head_dim (multiple of 8)");
  const bool record = g_profile.enabled && g_profile.count < g_profile.capacity;
  if (record) cudaEventRecord(g_profile.start[g_profile.count], stream);
  const int rc = run_attention_kernels(p, stream);
  if (record) cudaEventRecord(g_profile.stop[g_profile.count++], stream);
  return rc;
}

int run_attention_kernels(const AttnParams& p, cudaStream_t stream) {
  if (tc_eligible(p)) {
    int rc = p.kv_dtype == CG_F16 ? dispatch_tc<__half>(p, stream) : dispatch_tc<__nv_bfloat16>(p, stream);
    if (rc >= 0) return rc;
  }
  const int64_t items = p.batch * p.heads * p.steps;
  int64_t blocks = (items + 3) / 4;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  attn_simt_kernel<<<static_cast<unsigned>(blocks), 128, 0, stream>>>(p);
  return check_launch("attn_simt_kernel");
}

}  // namespace cg

extern "C" int cg_decode_attention(const void* q, int q_dtype, const void* k_cache, const void* v_cache, int kv_dtype,
                                   int64_t kv_stride_row, int64_t kv_stride_head, int64_t kv_stride_pos,
                                   const int64_t* rows, const int64_t* lengths, int64_t batch, int heads, int kv_heads,
                                   int steps, int head_dim, int span, float scale, void* out, int out_dtype,
                                   void* stream) {
  using namespace cg;
  CG_REQUIRE(batch >= 0 && heads > 0 && kv_heads > 0 && steps > 0 && head_dim > 0, "cg_decode_attention: bad shape");
  CG_REQUIRE(heads % kv_heads == 0, "cg_decode_attention: kv_heads %d must divide heads %d", kv_heads, heads);
  CG_REQUIRE(head_dim <= kSimtMaxDim, "cg_decode_attention: head_dim %d > %d", head_dim, kSimtMaxDim);
  CG_REQUIRE(valid_dtype(q_dtype) && valid_dtype(kv_dtype) && valid_dtype(out_dtype), "cg_decode_attention: bad dtype");
  CG_REQUIRE(span >= 0, "cg_decode_attention: negative span");
  if (batch == 0) return CG_OK;
  CG_REQUIRE(q && k_cache && v_cache && lengths && out, "cg_decode_attention: NULL pointer");
  AttnParams p{};
  p.q = q;
  p.q_dtype = q_dtype;
  p.q_st = head_dim;
  p.q_sh = static_cast<int64_t>(steps) * head_dim;
  p.q_sb = static_cast<int64_t>(heads) * steps * head_dim;
  p.k = k_cache;
  p.v = v_cache;
  p.kv_dtype = kv_dtype;
  p.kv_row = kv_stride_row;
  p.kv_head = kv_stride_head;
  p.kv_pos = kv_stride_pos;
  p.rows = rows;
  p.lengths = lengths;
  p.batch = batch;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.steps = steps;
  p.group = heads / kv_heads;
  p.head_dim = head_dim;
  p.span = span;
  p.scale = scale;
  p.out = out;
  p.out_dtype = out_dtype;
  p.o_sb = p.q_sb;
  p.o_sh = p.q_sh;
  p.o_st = p.q_st;
  return run_attention(p, static_cast<cudaStream_t>(stream));
}

extern "C" int cg_attention_profiling(int enable, int capacity) { return cg::profile_attention(enable, capacity); }

extern "C" int cg_attention_timings(float* ms_out, int max_count) {
  if (!ms_out || max_count < 0) return -1;
  return cg::attention_timings(ms_out, max_count);
}
