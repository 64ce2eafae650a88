// Non-causal attention with head dim 128 on tcgen05, the consumer of the
// projections' head-major q / k / v: for head h and query row i,
//
//   o[i, 128h .. 128h + 127] = softmax(scale · q_i · K^T) · V
//
// the reference's run_attn over the joint rows of a block (src/ming-dit.cc:
// 1905-2039; q, k and v as its tr_rope / transpose leave them). One CTA per
// (128-query tile, head), single-CTA MMAs (cta_group::1, M = 128):
//   * warp 0 loads Q once and K_j, V_j (128 keys each) per step with TMA into
//     two-stage rings (K and V released separately, K as soon as S_j is done);
//   * warp 1 issues S_j = Q · K_j^T into one of two TMEM S buffers, then
//     O_{j-1} = P_{j-1} · V_{j-1} into one of two TMEM O buffers (V as an
//     MN-major operand straight from its [keys][head dim] tile);
//   * warps 2-5 (thread = query row, TMEM lane) run the online softmax: a
//     first pass over S_j for the row maximum, a second for p = 2^(s·c − m)
//     (c = scale·log2 e), the row sum and P_j in bf16 (the PV operand, stored
//     128-byte swizzled), and fold each finished O_t into registers
//     (o = o · 2^(m_{t-1} − m_t) + O_t) once its buffer is complete;
//   * the epilogue divides by the row sum and stores bf16 rows token-major.
// S and P are double-buffered, so the softmax of tile j overlaps the MMAs
// of tiles j + 1 (S) and j - 1 (PV). Keys past S are masked (their tiles read
// zeros); rows past S are computed and not stored. Every wait is bounded;
// on a timeout the CTA unwinds and reports MP_ETIMEOUT.
#include <cuda_runtime.h>

#include "mp_device.cuh"
#include "mp_kernels.h"

namespace mp {

namespace {

constexpr int kAttnTile = 128;                          // query rows per CTA, keys per step
constexpr uint32_t kAttnBlk = 128 * 64 * 2;             // [128 rows][64 bf16], one TMA box
constexpr uint32_t kAttnOp = 2 * kAttnBlk;              // 128 rows x 128 bf16
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kAttnOp;             // K ring [2]
constexpr uint32_t kOffV = kOffK + 2 * kAttnOp;         // V ring [2]
constexpr uint32_t kOffP = kOffV + 2 * kAttnOp;         // P [2]
constexpr uint32_t kAttnTiles = kOffP + 2 * kAttnOp;    // 224 KB
constexpr uint32_t kAttnSmem = kAttnTiles + 1024 + 256;
static_assert(kAttnSmem <= 232448, "shared memory per CTA");
constexpr int kAttnThreads = 192;
constexpr uint32_t kAttnCols = 512;                     // S[0] S[1] O[0] O[1], 128 columns each

enum : uint32_t { kAttnSiteWait = 0x2100u, kAttnSiteDrain = 0x2200u };

struct AttnSmem {
  uint8_t* tiles;
  uint64_t* q_full;
  uint64_t* k_full;   // [2]
  uint64_t* k_empty;  // [2]
  uint64_t* v_full;   // [2]
  uint64_t* v_empty;  // [2]
  uint64_t* s_full;   // [2]
  uint64_t* s_free;   // [2]
  uint64_t* p_full;   // [2]
  uint64_t* o_full;   // [2]
  uint64_t* o_free;   // [2]
  uint64_t* drain;
  uint32_t* tmem_slot;
  volatile uint32_t* abort;
};

__device__ __forceinline__ AttnSmem carve_attn(uint8_t* raw) {
  AttnSmem s;
  const uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 1023u) & ~uintptr_t(1023u);
  s.tiles = reinterpret_cast<uint8_t*>(base);
  uint64_t* b = reinterpret_cast<uint64_t*>(s.tiles + kAttnTiles);
  s.q_full = b;
  s.k_full = b + 1;
  s.k_empty = b + 3;
  s.v_full = b + 5;
  s.v_empty = b + 7;
  s.s_full = b + 9;
  s.s_free = b + 11;
  s.p_full = b + 13;
  s.o_full = b + 15;
  s.o_free = b + 17;
  s.drain = b + 19;
  s.tmem_slot = reinterpret_cast<uint32_t*>(b + 20);
  s.abort = s.tmem_slot + 1;
  return s;
}

// K-major operand (128 rows x 128 bf16 as two [128][64] 128-byte-swizzled
// blocks): the 16-wide K step kk sits in block kk / 4 at byte 32 (kk % 4).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile, int kk) {
  return make_sdesc_sw128(tile + static_cast<uint32_t>(kk >> 2) * kAttnBlk +
                          static_cast<uint32_t>(kk & 3) * 32u);
}

// V as the MN-major B operand of P · V: its tile is [128 keys][128 head dims]
// as two [128 keys][64 dims] 128-byte-swizzled blocks, i.e. 8-key x 64-dim
// swizzle atoms of 1024 bytes. A 16-key step starts 2048 bytes further; the
// second 64-dim half lies one block (LBO) away; 8-key groups are 1024 bytes
// apart (SBO).
__device__ __forceinline__ uint64_t vmn_desc(uint32_t tile, int kk) {
  uint64_t d = 0;
  const uint32_t a = tile + static_cast<uint32_t>(kk) * 2048u;
  d |= static_cast<uint64_t>((a & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(kAttnBlk >> 4) << 16;  // leading byte offset: the next 64 dims
  d |= static_cast<uint64_t>(1024u >> 4) << 32;     // stride byte offset: the next 8 keys
  d |= static_cast<uint64_t>(1u) << 46;             // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;             // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ bool attn_wait(const AttnSmem& sm, uint64_t* bar, uint32_t parity,
                                          uint64_t limit) {
  return mbar_wait(smem_u32(bar), parity, sm.abort, kAttnSiteWait, limit);
}

// Warp 0, one thread.
__device__ void attn_producer(const AttnParams& p, const AttnSmem& sm, int q0, int head, int n) {
  const uint32_t base = smem_u32(sm.tiles);
  mbar_arrive_expect_tx(smem_u32(sm.q_full), kAttnOp);
  tma_load_3d(base + kOffQ, &p.tm_q, smem_u32(sm.q_full), 0, q0, head);
  tma_load_3d(base + kOffQ + kAttnBlk, &p.tm_q, smem_u32(sm.q_full), 64, q0, head);
  for (int j = 0; j < n; ++j) {
    const int b = j & 1;
    const uint32_t free_ph = static_cast<uint32_t>((j - 2) >> 1) & 1u;
    if (j >= 2 && !attn_wait(sm, &sm.k_empty[b], free_ph, p.wait_limit_ns)) return;
    const uint32_t kb = base + kOffK + static_cast<uint32_t>(b) * kAttnOp;
    mbar_arrive_expect_tx(smem_u32(&sm.k_full[b]), kAttnOp);
    tma_load_3d(kb, &p.tm_k, smem_u32(&sm.k_full[b]), 0, j * kAttnTile, head);
    tma_load_3d(kb + kAttnBlk, &p.tm_k, smem_u32(&sm.k_full[b]), 64, j * kAttnTile, head);
    if (j >= 2 && !attn_wait(sm, &sm.v_empty[b], free_ph, p.wait_limit_ns)) return;
    const uint32_t vb = base + kOffV + static_cast<uint32_t>(b) * kAttnOp;
    mbar_arrive_expect_tx(smem_u32(&sm.v_full[b]), kAttnOp);
    tma_load_3d(vb, &p.tm_v, smem_u32(&sm.v_full[b]), 0, j * kAttnTile, head);
    tma_load_3d(vb + kAttnBlk, &p.tm_v, smem_u32(&sm.v_full[b]), 64, j * kAttnTile, head);
  }
}

// Warp 1, one thread.
__device__ void attn_mma(const AttnParams& p, const AttnSmem& sm, uint32_t tmem, int n) {
  const uint32_t base = smem_u32(sm.tiles);
  const uint32_t idesc_qk = make_idesc_bf16(kAttnTile, kAttnTile);
  const uint32_t idesc_pv = idesc_qk | (1u << 16);  // B (V) MN-major
  bool ok = attn_wait(sm, sm.q_full, 0, p.wait_limit_ns);
  auto issue_s = [&](int j) -> bool {
    const int b = j & 1;
    if (!attn_wait(sm, &sm.k_full[b], static_cast<uint32_t>(j >> 1) & 1u, p.wait_limit_ns))
      return false;
    if (j >= 2 &&
        !attn_wait(sm, &sm.s_free[b], static_cast<uint32_t>((j - 2) >> 1) & 1u, p.wait_limit_ns))
      return false;
    tc_fence_after();
    const uint32_t kt = base + kOffK + static_cast<uint32_t>(b) * kAttnOp;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      umma_ss(tmem + static_cast<uint32_t>(b) * 128u, kmajor_desc(base + kOffQ, kk),
              kmajor_desc(kt, kk), idesc_qk, kk > 0 ? 1u : 0u);
    umma_commit(smem_u32(&sm.s_full[b]));
    umma_commit(smem_u32(&sm.k_empty[b]));
    return true;
  };
  auto issue_pv = [&](int t) -> bool {
    const int b = t & 1;
    const uint32_t ph = static_cast<uint32_t>(t >> 1) & 1u;
    if (!attn_wait(sm, &sm.v_full[b], ph, p.wait_limit_ns)) return false;
    if (!attn_wait(sm, &sm.p_full[b], ph, p.wait_limit_ns)) return false;
    if (t >= 2 &&
        !attn_wait(sm, &sm.o_free[b], static_cast<uint32_t>((t - 2) >> 1) & 1u, p.wait_limit_ns))
      return false;
    tc_fence_after();
    const uint32_t pt = base + kOffP + static_cast<uint32_t>(b) * kAttnOp;
    const uint32_t vt = base + kOffV + static_cast<uint32_t>(b) * kAttnOp;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      umma_ss(tmem + 256u + static_cast<uint32_t>(b) * 128u, kmajor_desc(pt, kk), vmn_desc(vt, kk),
              idesc_pv, kk > 0 ? 1u : 0u);
    umma_commit(smem_u32(&sm.o_full[b]));
    umma_commit(smem_u32(&sm.v_empty[b]));
    return true;
  };
  if (ok) ok = issue_s(0);
  for (int j = 1; ok && j < n; ++j) ok = issue_s(j) && issue_pv(j - 1);
  if (ok) ok = issue_pv(n - 1);
  // every MMA issued has completed before TMEM is freed
  umma_commit(smem_u32(sm.drain));
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(smem_u32(sm.drain), 0)) {
    if (global_timer_ns() - t0 > p.wait_limit_ns) {
      atomicCAS(const_cast<uint32_t*>(sm.abort), 0u, kAttnSiteDrain);
      break;
    }
  }
}

// Warps 2-5: thread = query row (TMEM lane).
__device__ void attn_softmax(const AttnParams& p, const AttnSmem& sm, uint32_t tmem, int q0,
                             int head, int n) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;
  const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
  const uint32_t swz = static_cast<uint32_t>(row & 7);
  const uint32_t pbase = smem_u32(sm.tiles) + kOffP + static_cast<uint32_t>(row) * 128u;
  const float c = p.scale_log2;
  float o[128];
#pragma unroll
  for (int d = 0; d < 128; ++d) o[d] = 0.0f;
  float m_run = -INFINITY, l = 0.0f;
  float a_m1 = 0.0f, a_m2 = 0.0f;  // alpha of tiles j-1 and j-2
  bool ok = true;
  // o = o * alpha + O_t (buffer t % 2)
  auto fold = [&](int t, float alpha) -> bool {
    const int b = t & 1;
    bool w = attn_wait(sm, &sm.o_full[b], static_cast<uint32_t>(t >> 1) & 1u, p.wait_limit_ns);
    if (!__all_sync(0xFFFFFFFFu, w)) return false;
    tc_fence_after();
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
      uint32_t v[32];
      MP_TMEM_LD_32X32B_X32(tmem + lane_base + 256u + static_cast<uint32_t>(b) * 128u +
                                static_cast<uint32_t>(32 * c4),
                            v);
      MP_TMEM_WAIT_LD_REGS32(v);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) o[32 * c4 + jj] = fmaf(o[32 * c4 + jj], alpha, __uint_as_float(v[jj]));
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&sm.o_free[b]));
    return true;
  };
  for (int j = 0; j < n && ok; ++j) {
    const int b = j & 1;
    bool w = attn_wait(sm, &sm.s_full[b], static_cast<uint32_t>(j >> 1) & 1u, p.wait_limit_ns);
    if (!__all_sync(0xFFFFFFFFu, w)) {
      ok = false;
      break;
    }
    tc_fence_after();
    const uint32_t sb = tmem + lane_base + static_cast<uint32_t>(b) * 128u;
    const int valid = p.S - j * kAttnTile;  // keys of this tile below S (>= 1)
    // pass 1: the row maximum
    float mx = -INFINITY;
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
      uint32_t v[32];
      MP_TMEM_LD_32X32B_X32(sb + static_cast<uint32_t>(32 * c4), v);
      MP_TMEM_WAIT_LD_REGS32(v);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj)
        if (32 * c4 + jj < valid) mx = fmaxf(mx, __uint_as_float(v[jj]));
    }
    const float m_new = fmaxf(m_run, mx * c);
    const float alpha = ex2(m_run - m_new);
    m_run = m_new;
    // P buffer b is free once O_{j-2} is complete; fold it first
    if (j >= 2 && !fold(j - 2, a_m2)) {
      ok = false;
      break;
    }
    // pass 2: p = 2^(s c - m), the row sum, P_j in bf16 (128-byte swizzled rows)
    float sum = 0.0f;
    const uint32_t prow = pbase + static_cast<uint32_t>(b) * kAttnOp;
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
      uint32_t v[32];
      MP_TMEM_LD_32X32B_X32(sb + static_cast<uint32_t>(32 * c4), v);
      MP_TMEM_WAIT_LD_REGS32(v);
      uint32_t w16[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int key = 32 * c4 + 2 * i;
        const float p0 = key < valid ? ex2(fmaf(__uint_as_float(v[2 * i]), c, -m_new)) : 0.0f;
        const float p1 = key + 1 < valid ? ex2(fmaf(__uint_as_float(v[2 * i + 1]), c, -m_new)) : 0.0f;
        sum += p0 + p1;
        w16[i] = pack_bf16x2(p0, p1);
      }
      const uint32_t blk = prow + static_cast<uint32_t>(c4 >> 1) * kAttnBlk;
#pragma unroll
      for (int i4 = 0; i4 < 4; ++i4) {
        const uint32_t ch = static_cast<uint32_t>((c4 & 1) * 4 + i4);
        st_shared_v4(blk + ((ch ^ swz) << 4), w16[4 * i4], w16[4 * i4 + 1], w16[4 * i4 + 2],
                     w16[4 * i4 + 3]);
      }
    }
    l = l * alpha + sum;
    tc_fence_before();  // S_j read out
    fence_proxy_async_shared();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(smem_u32(&sm.s_free[b]));
      mbar_arrive(smem_u32(&sm.p_full[b]));
    }
    a_m2 = a_m1;
    a_m1 = alpha;
  }
  if (ok && n >= 2) ok = fold(n - 2, a_m2);
  if (ok) ok = fold(n - 1, a_m1);
  if (!ok) return;
  const int q = q0 + row;
  if (q >= p.S) return;
  const float inv = 1.0f / l;
  uint16_t* dst = p.o + static_cast<size_t>(q) * p.ldo + static_cast<size_t>(head) * 128;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    uint4 w;
    w.x = pack_bf16x2(o[8 * i] * inv, o[8 * i + 1] * inv);
    w.y = pack_bf16x2(o[8 * i + 2] * inv, o[8 * i + 3] * inv);
    w.z = pack_bf16x2(o[8 * i + 4] * inv, o[8 * i + 5] * inv);
    w.w = pack_bf16x2(o[8 * i + 6] * inv, o[8 * i + 7] * inv);
    *reinterpret_cast<uint4*>(dst + 8 * i) = w;
  }
}

__global__ void __launch_bounds__(kAttnThreads, 1) attn_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  const AttnSmem sm = carve_attn(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q0 = static_cast<int>(blockIdx.x) * kAttnTile;
  const int head = static_cast<int>(blockIdx.y);
  const int n = (p.S + kAttnTile - 1) / kAttnTile;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(sm.q_full), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&sm.k_full[b]), 1);
      mbar_init(smem_u32(&sm.k_empty[b]), 1);
      mbar_init(smem_u32(&sm.v_full[b]), 1);
      mbar_init(smem_u32(&sm.v_empty[b]), 1);
      mbar_init(smem_u32(&sm.s_full[b]), 1);
      mbar_init(smem_u32(&sm.s_free[b]), 4);  // one arrive per softmax warp
      mbar_init(smem_u32(&sm.p_full[b]), 4);
      mbar_init(smem_u32(&sm.o_full[b]), 1);
      mbar_init(smem_u32(&sm.o_free[b]), 4);
    }
    mbar_init(smem_u32(sm.drain), 1);
    *sm.abort = 0u;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&p.tm_q);
    tma_prefetch_map(&p.tm_k);
    tma_prefetch_map(&p.tm_v);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(sm.tmem_slot), kAttnCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_slot;
  if (warp == 0) {
    if (lane == 0) attn_producer(p, sm, q0, head, n);
  } else if (warp == 1) {
    if (lane == 0) attn_mma(p, sm, tmem, n);
  } else {
    attn_softmax(p, sm, tmem, q0, head, n);
  }
  if (*sm.abort != 0u) {
    // error path only: let copies issued before the abort land before leaving
    const uint64_t t_settle = global_timer_ns();
    while (global_timer_ns() - t_settle < 100000ull) __nanosleep(1000);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kAttnCols);
  if (threadIdx.x == 0 && *sm.abort != 0u) atomicOr(p.err, kErrTimeout);
}

bool g_attn_configured[64] = {};

}  // namespace

cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!g_attn_configured[dev]) {
    e = cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kAttnSmem));
    if (e != cudaSuccess) return e;
    g_attn_configured[dev] = true;
  }
  const dim3 grid(static_cast<unsigned>((p.S + kAttnTile - 1) / kAttnTile),
                  static_cast<unsigned>(p.NH), 1);
  attn_kernel<<<grid, kAttnThreads, kAttnSmem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace mp
