// Ragged GQA decode attention straight from the KV pool.
//
// Reference: cardgym/nn/cuda_decode.py:46-151 (kernel + op) and the PyTorch path it
// short-cuts, cardgym/nn/trunk.py:203-256. Row b appends T tokens at its own length;
// query t of row b sees keys < min(lengths[b] + t, span). The merged query axis of
// a KV head is g * T + t (trunk.py:243-254).
//
// Two kernels:
//  * attn_tc: fp16/bf16 caches, head_dim in {16, 24, 32, 40, 48, 64}, G <= 16. One
//    warp per unit, persistent over units. A unit is a (row, KV head) pair and a block of
//    its steps: all T of them when G*T <= 16 (the decode case: one m16 tile of queries),
//    else floor(16 / G) steps per block (a prefill of T = 16 at G = 5: six blocks of three
//    steps, the same keys read from L2 by each). Each warp streams its units'
//    keys in chunks of 32 through a four-stage shared-memory ring filled with 16-byte
//    cp.async copies (zero-filled past the row's length, L2 evict-first; a unit's query
//    rows travel with its first chunk), computes Q K^T
//    and P V with mma.sync m16n8k16/k8 (fp32 accumulation) and keeps an online softmax
//    in fp32. Bulk-engine copies (cp.async.bulk) were measured to cost ~0.13 us each on
//    this part whatever their size below 16 KB, which capped 3 KB K/V chunks near
//    3.4 TB/s chip-wide; per-lane copies have no such per-copy cost.
//  * attn_simt: any cache dtype and shape; one warp per (row, query head, step),
//    fp32 arithmetic. Used for fp32 caches (the strict-parity mode) and shapes the
//    tensor-core kernel does not take.
#include "launch_timer.cuh"
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
constexpr int kChunk = 32;   // keys per staged chunk
constexpr int kStages = 4;   // chunk stages per warp: one computed while three load
constexpr int kTcWarps = 4;  // warps per CTA

__device__ __forceinline__ uint32_t smem_addr(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

// The KV stream is read once per layer: evict it from L2 first so that weights stay resident.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// One 16-byte asynchronous copy global -> shared; valid == false writes 16 zero bytes and reads nothing.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid, uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 16 : 0), "l"(policy)
               : "memory");
}

// Same, always copying 16 bytes.
__device__ __forceinline__ void cp_async16_full(void* dst, const void* src, uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "l"(policy)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
struct MmaOps;

template <>
struct MmaOps<__half> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t w) {
    return __half22float2(*reinterpret_cast<__half2*>(&w));
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
  static __device__ __forceinline__ float2 unpack(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w));
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

__device__ __forceinline__ void ldmatrix_x1(uint32_t& r0, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x1.shared.b16 {%0}, [%1];" : "=r"(r0) : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x2(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename KV, int D, bool kHalf>
struct TcShape {
  static constexpr int kTiles = D / 16;          // full k16 blocks of Q K^T
  static constexpr bool kTail = (D % 16) != 0;   // one trailing k8 block
  static constexpr int kDTiles = D / 8;          // n8 tiles of the output
  static constexpr int kPieces = D / 8;          // 16-byte pieces per key (or query) row
  static constexpr int kQRows = kHalf ? 8 : 16;  // query rows staged (rows >= G*T zero-filled)
  static constexpr int kChunkElems = kChunk * D; // per K or V
  static constexpr int kStageElems = 2 * kChunkElems + kQRows * D;  // K, V, then the unit's q
  static constexpr int kWarpBytes = kStages * kStageElems * static_cast<int>(sizeof(KV));
};

// Steps per unit: every step when the G*T query rows fit one m16 tile, else the most that do.
__host__ __device__ inline int step_block(int group, int steps) { return group * steps <= 16 ? steps : 16 / group; }

// Rows with no visible key get a zero output: the unit's steps t0 .. t0 + tb - 1.
__device__ void zero_unit(const AttnParams& p, int64_t b, int kvh, int t0, int tb, int lane) {
  const int D = p.head_dim;
  for (int i = lane; i < p.group * tb * D; i += 32) {
    const int m = i / D, d = i % D;
    const int h = kvh * p.group + m / tb, t = t0 + m % tb;
    const int64_t off = p.out_blocked ? blocked_offset(b * p.steps + t, h * D + d, p.blocked_width)
                                      : b * p.o_sb + h * p.o_sh + t * p.o_st + d;
    store_from_float(p.out, off, p.out_dtype, 0.f);
  }
}

// A claimed (row, KV head) unit: decoded once, handed from the issue cursor to the compute
// cursor through a small per-warp ring.
struct TcUnit {
  int b;     // batch index
  int kvh;   // KV head
  int keys;  // keys visible to the unit's last query (> 0)
  int len;   // min(lengths[b] + t0, span): keys visible to its first step
  int t0;    // its first step
};

constexpr int kRing = 8;  // units claimed ahead by the issue cursor, per warp

// kHalf: G * T <= 8, so rows 8..15 of the m16 tile are padding and are never processed.
// kBlocked: the output goes to the tile-blocked bf16 operand layout; otherwise it has the
// cache dtype and q's [B, H, T, D] strides.
template <typename KV, int D, bool kHalf, bool kBlocked>
__global__ void __launch_bounds__(kTcWarps * 32) attn_tc_kernel(AttnParams p) {
  using Shape = TcShape<KV, D, kHalf>;
  using Ops = MmaOps<KV>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int gid = lane >> 2, tid4 = lane & 3;
  KV* stage_base = reinterpret_cast<KV*>(smem_raw + wib * Shape::kWarpBytes);
  const uint64_t policy = evict_first_policy();
  // Zeroed stages: a block past a chunk's zero-filled keys then only ever holds finite data.
  for (int i = lane; i < Shape::kWarpBytes / 16; i += 32) reinterpret_cast<uint4*>(stage_base)[i] = make_uint4(0, 0, 0, 0);
  __syncwarp();
  pdl_wait();  // q, K and V come from the kernel before
  pdl_trigger();

  const int sblk = step_block(p.group, p.steps);
  const int nblk = (p.steps + sblk - 1) / sblk;
  const int units = static_cast<int>(p.batch * p.kv_heads * nblk);  // < 2^31: checked by the host
  const int M = p.group * sblk;  // query rows of a unit's tile (a short last block uses fewer)
  const float scale_log2 = p.scale * 1.4426950408889634f;
  const KV* kc = static_cast<const KV*>(p.k);
  const KV* vc = static_cast<const KV*>(p.v);
  const KV* qg = static_cast<const KV*>(p.q);

  // Units are claimed from p.counter (or by a static stride). The issue cursor runs
  // kStages - 1 chunks ahead of the compute cursor and passes each claimed unit on through
  // the ring. Units without visible keys get zero outputs when claimed.
  __shared__ int4 ring[kTcWarps][kRing];
  int static_next = blockIdx.x * kTcWarps + wib;
  const int stride = gridDim.x * kTcWarps;
  int head = 0, tail = 0;
  auto claim = [&](TcUnit& u) -> bool {
    while (true) {
      int x;
      if (p.counter) {
        int v = 0;
        if (lane == 0) v = atomicAdd(p.counter, 1);
        x = __shfl_sync(0xffffffffu, v, 0);
      } else {
        x = static_next;
        static_next += stride;
      }
      if (x >= units) return false;
      // Consecutive units are the step blocks of one (row, KV head): their keys stay in L2.
      const int per_row = p.kv_heads * nblk;
      const int b = x / per_row, rest = x - b * per_row;
      const int kvh = rest / nblk, t0 = (rest - kvh * nblk) * sblk;
      const int tb = min(sblk, p.steps - t0);
      const int64_t len = p.lengths[b] + t0;
      const int64_t last = len + tb - 1;
      const int keys = static_cast<int>(last < p.span ? last : p.span);
      if (keys <= 0) {
        zero_unit(p, b, kvh, t0, tb, lane);
        continue;
      }
      u.b = b;
      u.kvh = kvh;
      u.keys = keys;
      u.len = static_cast<int>(len < p.span ? len : p.span);
      u.t0 = t0;
      return true;
    }
  };

  // Per-lane constants of the launch: the query pieces this lane stages for every unit (offset
  // from the unit's first query row), and the step of the output rows it finalizes.
  constexpr int kQPieces = Shape::kQRows * Shape::kPieces;
  constexpr int kQIters = (kQPieces + 31) / 32;
  int q_off[kQIters];
  int q_t[kQIters];  // the piece's step within the unit's block
  bool q_ok[kQIters];
#pragma unroll
  for (int it = 0; it < kQIters; ++it) {
    const int i = lane + 32 * it;
    const int m = i / Shape::kPieces, piece = i - m * Shape::kPieces;
    q_ok[it] = i < kQPieces && m < M;
    q_t[it] = q_ok[it] ? m % sblk : 0;
    q_off[it] = q_ok[it] ? static_cast<int>((m / sblk) * p.q_sh + (m % sblk) * p.q_st) + piece * 8 : 0;
  }
  int row_h[2], row_t[2], row_tlim[2];  // rows gid and gid + 8: head within the group, step, step for the limit
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int m = gid + 8 * r;
    row_h[r] = m < M ? m / sblk : 0;
    row_t[r] = m < M ? m % sblk : 0;
    row_tlim[r] = m < M ? row_t[r] : sblk - 1;  // padding rows attend to every visible key: finite, never stored
  }

  // Issue cursor.
  bool issue_live = true;
  TcUnit iu{0, 0, 0, 0, 0};
  int issue_chunk_no = 0;
  int64_t issue_kv = 0;  // element offset of the unit's (row, KV head) block in the pool
  auto issue_next_unit = [&]() {
    issue_live = claim(iu);
    issue_chunk_no = 0;
    if (issue_live) {
      const int64_t row = p.rows ? p.rows[iu.b] : iu.b;
      issue_kv = row * p.kv_row + iu.kvh * p.kv_head;
    }
    // KV head and first step share one slot: kv_heads < 2^16 and steps < 2^15 (checked by the host).
    if (lane == 0) ring[wib][head % kRing] = issue_live ? make_int4(iu.b, iu.kvh | (iu.t0 << 16), iu.keys, iu.len)
                                                        : make_int4(0, 0, 0, -1);
    ++head;
  };
  // A chunk of K (and of V) is one contiguous range of n * D elements in the pool and in
  // the stage; lanes copy it in 16-byte pieces, zero-filled up to the 16-key MMA block.
  // A unit's first chunk also brings its query rows (rows >= G*T zero-filled).
  auto issue_chunk = [&](int stage) {
    if (issue_live) {
      const int first = issue_chunk_no * kChunk;
      const int n = min(kChunk, iu.keys - first);
      const int valid_pieces = n * Shape::kPieces;
      const int pieces = ((n + 15) & ~15) * Shape::kPieces;
      const uint4* ksrc = reinterpret_cast<const uint4*>(kc + issue_kv + static_cast<int64_t>(first) * D);
      const uint4* vsrc = reinterpret_cast<const uint4*>(vc + issue_kv + static_cast<int64_t>(first) * D);
      KV* sbase = stage_base + stage * Shape::kStageElems;
      uint4* kdst = reinterpret_cast<uint4*>(sbase) + lane;
      uint4* vdst = reinterpret_cast<uint4*>(sbase + Shape::kChunkElems) + lane;
      // Rounds of 32 pieces: whole rounds of valid keys copy without checks; the boundary
      // round zero-fills its lanes past the valid keys (source clamped to the chunk start).
      constexpr int kRounds = kChunk * Shape::kPieces / 32;
#pragma unroll
      for (int it = 0; it < kRounds; ++it) {
        if (32 * it >= pieces) break;
        if (32 * it + 32 <= valid_pieces) {
          cp_async16_full(kdst + 32 * it, ksrc + lane + 32 * it, policy);
          cp_async16_full(vdst + 32 * it, vsrc + lane + 32 * it, policy);
        } else {
          const int i = lane + 32 * it;
          const bool valid = i < valid_pieces;
          cp_async16(kdst + 32 * it, ksrc + (valid ? i : 0), valid, policy);
          cp_async16(vdst + 32 * it, vsrc + (valid ? i : 0), valid, policy);
        }
      }
      if (issue_chunk_no == 0) {
        uint4* qdst = reinterpret_cast<uint4*>(sbase + 2 * Shape::kChunkElems) + lane;
        const KV* qunit = qg + iu.b * p.q_sb + static_cast<int64_t>(iu.kvh) * p.group * p.q_sh +
                          static_cast<int64_t>(iu.t0) * p.q_st;
#pragma unroll
        for (int it = 0; it < kQIters; ++it) {
          // Rows past the last step (a short last block) are zero-filled like the tile's padding.
          const bool ok = q_ok[it] && iu.t0 + q_t[it] < p.steps;
          if (lane + 32 * it < kQPieces) cp_async16(qdst + 32 * it, qunit + (ok ? q_off[it] : 0), ok, policy);
        }
      }
    }
    cp_async_commit();  // one group per chunk slot, empty or not: keeps the group count in step
  };
  auto issue_advance = [&]() {
    if (!issue_live) return;
    if (++issue_chunk_no * kChunk < iu.keys) return;
    issue_next_unit();
  };

  issue_next_unit();
  int issue_stage = 0;
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    issue_chunk(issue_stage);
    issue_advance();
    issue_stage = issue_stage + 1 == kStages ? 0 : issue_stage + 1;
  }

  // Compute cursor.
  auto pop = [&](TcUnit& u) -> bool {
    __syncwarp();
    const int4 r = ring[wib][tail % kRing];
    ++tail;
    u.b = r.x;
    u.kvh = r.y & 0xffff;
    u.t0 = r.y >> 16;
    u.keys = r.z;
    u.len = r.w;
    return r.w >= 0;
  };
  TcUnit cu;
  bool comp_live = pop(cu);
  int comp_chunk = 0;

  uint32_t qa[Shape::kTiles > 0 ? Shape::kTiles : 1][4];
  uint32_t qt[2] = {0, 0};
  float o[Shape::kDTiles][4];
  float mrow[2], lrow[2];
  int limit_r[2];
  int comp_stage = 0;
  constexpr int kRows = kHalf ? 1 : 2;

  while (comp_live) {
    issue_chunk(issue_stage);
    issue_advance();
    issue_stage = issue_stage + 1 == kStages ? 0 : issue_stage + 1;

    cp_async_wait<kStages - 1>();
    __syncwarp();
    const KV* ks = stage_base + comp_stage * Shape::kStageElems;
    const KV* vs = ks + Shape::kChunkElems;
    if (comp_chunk == 0) {
      // Unit start: Q fragments from the stage, softmax state, limits.
      const KV* qs = ks + 2 * Shape::kChunkElems;
#pragma unroll
      for (int kb = 0; kb < Shape::kTiles; ++kb) {
        if (kHalf) {
          ldmatrix_x2(qa[kb][0], qa[kb][2], smem_addr(qs + (lane & 7) * D + kb * 16 + ((lane >> 3) & 1) * 8));
          qa[kb][1] = qa[kb][3] = 0u;
        } else {
          ldmatrix_x4(qa[kb][0], qa[kb][1], qa[kb][2], qa[kb][3],
                      smem_addr(qs + (lane & 15) * D + kb * 16 + (lane >> 4) * 8));
        }
      }
      if (Shape::kTail) {
        if (kHalf) {
          ldmatrix_x1(qt[0], smem_addr(qs + (lane & 7) * D + Shape::kTiles * 16));
          qt[1] = 0u;
        } else {
          ldmatrix_x2(qt[0], qt[1], smem_addr(qs + (lane & 15) * D + Shape::kTiles * 16));
        }
      }
#pragma unroll
      for (int j = 0; j < Shape::kDTiles; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        limit_r[r] = min(cu.len + row_tlim[r], p.span);
        mrow[r] = -INFINITY;
        lrow[r] = 0.f;
      }
    }

    const int first = comp_chunk * kChunk;
    const int n = min(kChunk, cu.keys - first);
    // Every 16-key block of the chunk is processed (no per-block branches); a chunk that is
    // partial, or whose keys some row does not see yet, is masked, so keys past the unit's end
    // (zero-filled, or finite data from an earlier chunk: the stages start zeroed) get p = 0.
    const bool full = n == kChunk && first + n <= cu.len;
    // S = Q K^T over the chunk, 16 keys (two n8 tiles) per step; K fragments by ldmatrix.
    // Scores stay unscaled until the exponent: scale > 0 keeps the max where it is.
    float s[kChunk / 8][4];
    float kmax[kChunk / 16][2];  // per 16-key block, then a tree: no long max chain
#pragma unroll
    for (int kk = 0; kk < kChunk / 16; ++kk) {
      kmax[kk][0] = kmax[kk][1] = -INFINITY;
      float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
      {
        const KV* kbase = ks + (kk * 16 + (lane & 15)) * D;
#pragma unroll
        for (int kb = 0; kb < Shape::kTiles; ++kb) {
          uint32_t r0, r1, r2, r3;
          ldmatrix_x4(r0, r1, r2, r3, smem_addr(kbase + kb * 16 + (lane >> 4) * 8));
          Ops::k16(acc0, qa[kb], r0, r2);
          Ops::k16(acc1, qa[kb], r1, r3);
        }
        if (Shape::kTail) {
          uint32_t r0, r1;
          ldmatrix_x2(r0, r1, smem_addr(kbase + Shape::kTiles * 16));
          Ops::k8(acc0, qt[0], qt[1], r0);
          Ops::k8(acc1, qt[0], qt[1], r1);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s[2 * kk][e] = -INFINITY;
        s[2 * kk + 1][e] = -INFINITY;
      }
      {
#pragma unroll
        for (int e = 0; e < 2 * kRows; ++e) {
          const int r = e >> 1;
          float v0 = acc0[e], v1 = acc1[e];
          if (!full) {
            const int key = first + kk * 16 + 2 * tid4 + (e & 1);
            v0 = key < limit_r[r] ? v0 : -INFINITY;
            v1 = key + 8 < limit_r[r] ? v1 : -INFINITY;
          }
          s[2 * kk][e] = v0;
          s[2 * kk + 1][e] = v1;
          kmax[kk][r] = fmaxf(kmax[kk][r], fmaxf(v0, v1));
        }
      }
    }
    float cmax[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
#pragma unroll
      for (int w = kChunk / 32; w >= 1; w /= 2)
#pragma unroll
        for (int kk = 0; kk < w; ++kk) kmax[kk][r] = fmaxf(kmax[kk][r], kmax[kk + w][r]);
      cmax[r] = kmax[0][r];
    }
    float alpha[2] = {1.f, 1.f};
    float psum[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // two partial sums per row: shorter add chains
    float neg_max[2];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      cmax[r] = fmaxf(cmax[r], __shfl_xor_sync(0xffffffffu, cmax[r], 1));
      cmax[r] = fmaxf(cmax[r], __shfl_xor_sync(0xffffffffu, cmax[r], 2));
      const float m_new = fmaxf(mrow[r], cmax[r] * scale_log2);  // running max, in log2 units
      // A row with no visible key so far keeps m = -inf: its scores are all -inf, so any
      // finite offset gives p = 0, and its (zero) accumulators need no rescaling.
      const bool empty = m_new == -INFINITY;
      alpha[r] = empty ? 1.f : fast_exp2(mrow[r] - m_new);  // exp2(-inf) = 0 on the first chunk
      mrow[r] = m_new;
      neg_max[r] = empty ? 0.f : -m_new;
    }
#pragma unroll
    for (int j = 0; j < kChunk / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2 * kRows; ++e) {
        const int r = e >> 1;
        const float pe = fast_exp2(fmaf(s[j][e], scale_log2, neg_max[r]));  // masked keys: exp2(-inf) = 0
        s[j][e] = pe;
        psum[r][j & 1] += pe;
      }
    }
#pragma unroll
    for (int r = 0; r < kRows; ++r) lrow[r] = lrow[r] * alpha[r] + (psum[r][0] + psum[r][1]);
#pragma unroll
    for (int j = 0; j < Shape::kDTiles; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      if (!kHalf) {
        o[j][2] *= alpha[1];
        o[j][3] *= alpha[1];
      }
    }

    // O += P V, 16 keys at a time.
#pragma unroll
    for (int kk = 0; kk < kChunk / 16; ++kk) {
      {
        uint32_t pa[4];
        pa[0] = Ops::pack(s[2 * kk][0], s[2 * kk][1]);
        pa[1] = kHalf ? 0u : Ops::pack(s[2 * kk][2], s[2 * kk][3]);
        pa[2] = Ops::pack(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        pa[3] = kHalf ? 0u : Ops::pack(s[2 * kk + 1][2], s[2 * kk + 1][3]);
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
    __syncwarp();  // every lane is done with this stage before it is refilled

    const bool last_chunk = first + kChunk >= cu.keys;
    if (last_chunk) {
      // Unit done: normalise and store rows m < M.
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
      }
      const int64_t b = cu.b;
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        const int m = gid + 8 * r;
        if (m < M && cu.t0 + row_t[r] < p.steps) {
          const float inv = 1.f / lrow[r];
          const int h = cu.kvh * p.group + row_h[r], t = cu.t0 + row_t[r];
#pragma unroll
          for (int j = 0; j < Shape::kDTiles; ++j) {
            const int d = j * 8 + 2 * tid4;
            const float x0 = o[j][2 * r] * inv, x1 = o[j][2 * r + 1] * inv;
            if (kBlocked) {
              // even column pair inside one 8-column chunk: one 32-bit store of two bf16
              const int64_t off = blocked_offset(b * p.steps + t, h * D + d, p.blocked_width);
              *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(p.out) + off) =
                  __floats2bfloat162_rn(x0, x1);
            } else {
              KV* out = static_cast<KV*>(p.out) + b * p.o_sb + h * p.o_sh + t * p.o_st + d;
              *reinterpret_cast<uint32_t*>(out) = Ops::pack(x0, x1);
            }
          }
        }
      }
      comp_live = pop(cu);
      comp_chunk = 0;
    } else {
      ++comp_chunk;
    }
    comp_stage = comp_stage + 1 == kStages ? 0 : comp_stage + 1;
  }
  cp_async_wait<0>();  // no copy may still target shared memory when the warp exits
}

template <typename KV, int D, bool kHalf, bool kBlocked>
int launch_tc(const AttnParams& p, cudaStream_t stream) {
  using Shape = TcShape<KV, D, kHalf>;
  auto kernel = attn_tc_kernel<KV, D, kHalf, kBlocked>;
  const int smem = kTcWarps * Shape::kWarpBytes;
  static int per_sm[64] = {0};
  int device = 0;
  cudaGetDevice(&device);
  int& occupancy = per_sm[device & 63];
  if (!occupancy) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "attn_tc_kernel smem: %s", cudaGetErrorString(err));
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occupancy, kernel, kTcWarps * 32, smem);
    if (occupancy < 1) occupancy = 1;
  }
  const int sblk = step_block(p.group, p.steps);
  const int64_t units = p.batch * p.kv_heads * ((p.steps + sblk - 1) / sblk);
  int64_t blocks = static_cast<int64_t>(sm_count()) * occupancy;
  const int64_t needed = (units + kTcWarps - 1) / kTcWarps;
  if (blocks > needed) blocks = needed;
  if (blocks < 1) return CG_OK;
  return launch_pdl("attn_tc_kernel", kernel, dim3(static_cast<unsigned>(blocks)), dim3(kTcWarps * 32), smem, stream,
                    p);
}

template <typename KV, int D>
int dispatch_layout(const AttnParams& p, cudaStream_t stream) {
  const bool half = p.group * step_block(p.group, p.steps) <= 8;
  if (p.out_blocked) return half ? launch_tc<KV, D, true, true>(p, stream) : launch_tc<KV, D, false, true>(p, stream);
  return half ? launch_tc<KV, D, true, false>(p, stream) : launch_tc<KV, D, false, false>(p, stream);
}

template <typename KV>
int dispatch_tc(const AttnParams& p, cudaStream_t stream) {
  switch (p.head_dim) {
    case 16: return dispatch_layout<KV, 16>(p, stream);
    case 24: return dispatch_layout<KV, 24>(p, stream);
    case 32: return dispatch_layout<KV, 32>(p, stream);
    case 40: return dispatch_layout<KV, 40>(p, stream);
    case 48: return dispatch_layout<KV, 48>(p, stream);
    case 64: return dispatch_layout<KV, 64>(p, stream);
    default: return -1;
  }
}

bool tc_eligible(const AttnParams& p) {
  if (p.kv_dtype == CG_F32) return false;
  if (p.group > 16 || p.kv_heads >= (1 << 16) || p.steps >= (1 << 15)) return false;
  const int d = p.head_dim;
  if (!(d == 16 || d == 24 || d == 32 || d == 40 || d == 48 || d == 64)) return false;
  // q (and the non-blocked output) in the cache dtype; q rows are copied in 16-byte pieces,
  // the output is written in 32-bit pairs.
  if (p.q_dtype != p.kv_dtype) return false;
  if (!p.out_blocked && p.out_dtype != p.kv_dtype) return false;
  if ((p.q_sb | p.q_sh | p.q_st) & 7) return false;
  const int sblk = step_block(p.group, p.steps);
  if (p.batch * p.kv_heads * ((p.steps + sblk - 1) / sblk) >= (1LL << 31)) return false;
  if (!p.out_blocked && ((p.o_sb | p.o_sh | p.o_st) & 1)) return false;
  // 16-byte copies: contiguous key rows, aligned row/head strides and bases.
  if (p.kv_pos != d) return false;
  if ((p.kv_row % 8) || (p.kv_head % 8)) return false;
  if ((reinterpret_cast<uintptr_t>(p.k) & 15) || (reinterpret_cast<uintptr_t>(p.v) & 15)) return false;
  if (reinterpret_cast<uintptr_t>(p.q) & 15 || reinterpret_cast<uintptr_t>(p.out) & 3) return false;
  return true;
}

namespace {
LaunchTimer g_attention_timer;
}  // namespace

int profile_attention(int enable, int capacity) {
  return g_attention_timer.configure(enable, capacity, "cg_attention_profiling");
}

int attention_timings(float* ms_out, int max_count) { return g_attention_timer.timings(ms_out, max_count); }

int run_attention_kernels(const AttnParams& p, cudaStream_t stream);

int run_attention(const AttnParams& p, cudaStream_t stream) {
  if (p.batch == 0) return CG_OK;
  if (p.out_blocked && (p.out_dtype != CG_BF16 || p.blocked_width != p.heads * p.head_dim || p.blocked_width % 8))
    return set_error(CG_ERR_ARGUMENT, "blocked attention output must be bf16 with width heads*head_dim (multiple of 8)");
  const bool recorded = g_attention_timer.begin(stream);
  const int rc = run_attention_kernels(p, stream);
  g_attention_timer.end(stream, recorded);
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
