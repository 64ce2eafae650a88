// The fused projection kernel on CTA PAIRS (cluster of 2, tcgen05 cta_group::2):
//
//   y[M, N] = x[M, K] · deq(W)[N, K]^T  +  T[M, R] · Bstack[N, R]^T
//
// the reference's `lin` (src/ming-dit.cc:1763-1771) as one pass over K with
// the live LoRA slots appended as extra K tiles, on a tile of 256 output
// features x up to 256 tokens per pair of SMs. One launch may cover up to
// four projections of the same input (q/k/v, w1/w3): each pair maps to the
// member whose feature range it falls in.
//   * each CTA owns 128 of the pair's features (MMA M = 256 across the pair)
//     and loads HALF of the pair's token rows (MMA N is split across the
//     pair), so every SM streams half the activation bytes a single-CTA
//     128 x 256 tile needs, and a 64-wide K stage costs 32 KB of shared
//     memory: six stages fit;
//   * each CTA dequantizes its own 128 feature rows into its own TMEM (two
//     warpgroups, each converting half of the stage's 64 columns with packed
//     f32x2 arithmetic), and the leader's single MMA thread issues
//     tcgen05.mma.cta_group::2 reading both CTAs' TMEM A stages and shared B
//     halves;
//   * activation / dense-weight / LoRA tiles complete on the LEADER's full
//     barrier (cta_group::2 TMA); the codes tile of each CTA completes on
//     that CTA's own barrier, where its dequantizers wait; the MMA commit
//     multicasts stage release and accumulator-ready to both CTAs.
#include <cuda_runtime.h>

#include "mp_device.cuh"
#include "mp_kernels.h"

namespace mp {

namespace {

// Stage count and TMEM column placement (tunable at compile time for
// measurements; the defaults are the shipped configuration).
#ifndef MP_PAIR_STAGES
#define MP_PAIR_STAGES 6
#endif
#ifndef MP_ACOL_BASE
#define MP_ACOL_BASE 256
#endif
#ifndef MP_ACOL_STRIDE
#define MP_ACOL_STRIDE 32
#endif
#ifndef MP_ACC_BASE
#define MP_ACC_BASE 0
#endif
constexpr int kPairStages = MP_PAIR_STAGES;
constexpr int kPairXBytes = (kMaxTok / 2) * 128;       // this CTA's token rows: 16 KB
constexpr int kPairStageBytes = kPairXBytes + kWStageBytes;  // 32 KB
constexpr int kPairThreads = 320;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-9 dequant + epilogue
constexpr int kDeqThreads = 256;
constexpr int kPairACol = MP_ACOL_BASE;       // TMEM A stages
constexpr int kPairAStride = MP_ACOL_STRIDE;  // columns between A stages (32 used)
constexpr int kPairAcc = MP_ACC_BASE;         // f32 accumulator: n_tok columns
static_assert(kPairACol + (kPairStages - 1) * kPairAStride + 32 <= kTmemCols, "TMEM A stages");
constexpr uint32_t kPairSmemBytes = kPairStages * kPairStageBytes + 1024 + 512;

enum : uint32_t {
  kSiteEmpty = 0x1100u,
  kSiteFull = 0x1200u,
  kSiteDeq = 0x1300u,
  kSiteCodes = 0x1400u,
  kSiteEpi = 0x1500u,
  kSiteDrain = 0x1600u,
};

// Per-stage timeline of the first CTA pair, only in builds compiled with
// -DMP_TRACE (a profiling build; the product library has no trace code).
#ifdef MP_TRACE
constexpr int kTraceStages = 96;
enum { kTrProducer = 0, kTrDeqStart, kTrDeqEnd, kTrMma, kTrEpiStart, kTrEpiEnd, kTrDeqMath,
       kTrDeqStored, kTrEvents };
__device__ long long g_trace[2][kTrEvents][kTraceStages];
__device__ __forceinline__ void trace_mark(int ev, int kt) {
  if (blockIdx.x < 2 && blockIdx.y == 0 && kt < kTraceStages) g_trace[blockIdx.x][ev][kt] = clock64();
}
#define MP_TRACE_MARK(ev, kt) trace_mark(ev, kt)
#else
#define MP_TRACE_MARK(ev, kt) ((void)0)
#endif

struct PairSmem {
  uint8_t* tiles;
  uint64_t* full;    // [stages] leader: both CTAs' TMA tiles of the MMA
  uint64_t* empty;   // [stages] each CTA: stage released by the MMA
  uint64_t* cfull;   // [stages] each CTA: its own codes tile landed
  uint64_t* afull;   // [stages] leader: both CTAs' dequantized TMEM stage written
  uint64_t* tfull;   // each CTA: accumulator complete
  uint64_t* drain;   // leader: every MMA issued has completed
  uint32_t* tmem_slot;
  volatile uint32_t* abort;
};

__device__ __forceinline__ PairSmem carve_pair(uint8_t* raw) {
  PairSmem s;
  const uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 1023u) & ~uintptr_t(1023u);
  s.tiles = reinterpret_cast<uint8_t*>(base);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s.tiles + kPairStages * kPairStageBytes);
  s.full = bars;
  s.empty = bars + kPairStages;
  s.cfull = bars + 2 * kPairStages;
  s.afull = bars + 3 * kPairStages;
  s.tfull = bars + 4 * kPairStages;
  s.drain = s.tfull + 1;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.drain + 1);
  s.abort = s.tmem_slot + 1;
  return s;
}

// 4 packed 8-bit codes -> two bf16x2 words, with packed fp32 pairs.
__device__ __forceinline__ void deq8x4(uint32_t w, uint64_t magic2, uint64_t sc2, uint64_t bi2,
                                       uint32_t& p0, uint32_t& p1) {
  const uint64_t a = f32x2(__uint_as_float(__byte_perm(w, 0x4Bu, 0x4550u)),
                           __uint_as_float(__byte_perm(w, 0x4Bu, 0x4551u)));
  const uint64_t b = f32x2(__uint_as_float(__byte_perm(w, 0x4Bu, 0x4552u)),
                           __uint_as_float(__byte_perm(w, 0x4Bu, 0x4553u)));
  p0 = f32x2_to_bf16x2(fma_f32x2(add_f32x2(a, magic2), sc2, bi2));
  p1 = f32x2_to_bf16x2(fma_f32x2(add_f32x2(b, magic2), sc2, bi2));
}

// 8 packed 4-bit codes (code j at bits [4j, 4j+4)) -> four bf16x2 words.
__device__ __forceinline__ void deq4x8(uint32_t w, uint64_t magic2, uint64_t sc2, uint64_t bi2,
                                       uint32_t* p) {
  const uint32_t ev = w & 0x0F0F0F0Fu;          // codes 0, 2, 4, 6
  const uint32_t od = (w >> 4) & 0x0F0F0F0Fu;   // codes 1, 3, 5, 7
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t sel = 0x4550u | static_cast<uint32_t>(b);
    const uint64_t q = f32x2(__uint_as_float(__byte_perm(ev, 0x4Bu, sel)),
                             __uint_as_float(__byte_perm(od, 0x4Bu, sel)));
    p[b] = f32x2_to_bf16x2(fma_f32x2(add_f32x2(q, magic2), sc2, bi2));
  }
}

__device__ __forceinline__ uint32_t pick4p(const uint4& v, int i) {
  uint32_t r = v.x;
  r = (i == 1) ? v.y : r;
  r = (i == 2) ? v.z : r;
  r = (i == 3) ? v.w : r;
  return r;
}

__device__ void pair_producer(const ProjParams& p, const ProjMember& mb, const PairSmem& sm,
                              bool leader, int f0,
                              int tx0, int base_kt, int total_kt) {
  const bool quant = mb.bits != 0;
  const uint32_t half_rows = static_cast<uint32_t>(p.n_tok / 2);
  const uint32_t xbytes_pair = 2u * half_rows * 128u;
  const uint32_t codes_bytes = static_cast<uint32_t>(kBlockN * kBlockK * mb.bits / 8);
  int issued = 0;
  for (int kt = 0; kt < total_kt; ++kt) {
    const int s = kt % kPairStages;
    const uint32_t ph = static_cast<uint32_t>(kt / kPairStages) & 1u;
    if (kt >= kPairStages &&
        !mbar_wait(smem_u32(&sm.empty[s]), ph ^ 1u, sm.abort, kSiteEmpty | s, p.wait_limit_ns))
      break;
    MP_TRACE_MARK(kTrProducer, kt);
    const uint32_t xb = smem_u32(sm.tiles + s * kPairStageBytes);
    const uint32_t wb = xb + kPairXBytes;
    const uint32_t full_local = smem_u32(&sm.full[s]);
    const uint32_t full_leader = mapa_shared(full_local, 0);
    if (kt < base_kt && quant) {
      if (leader) mbar_arrive_expect_tx(full_local, xbytes_pair);
      tma_load_2d_pair(xb, &p.tm_x, full_leader, kt * kBlockK, tx0);
      const uint32_t cbar = smem_u32(&sm.cfull[s]);
      mbar_arrive_expect_tx(cbar, codes_bytes);
      tma_load_2d(wb, &mb.tm_w, cbar, kt * kBlockK * mb.bits / 8, f0);
    } else {
      if (leader) mbar_arrive_expect_tx(full_local, xbytes_pair + 2u * kWStageBytes);
      if (kt < base_kt) {
        tma_load_2d_pair(xb, &p.tm_x, full_leader, kt * kBlockK, tx0);
        tma_load_2d_pair(wb, &mb.tm_w, full_leader, kt * kBlockK, f0);
      } else {
        const int j = kt - base_kt;
        tma_load_2d_pair(xb, &mb.tm_t, full_leader, j * kBlockK, tx0);
        tma_load_2d_pair(wb, &mb.tm_b, full_leader, j * kBlockK, f0);
      }
    }
    issued = kt + 1;
  }
  if (*sm.abort != 0u) {
    // Unwind: wait (bounded) for this CTA's own codes copies still in flight;
    // the pair copies are drained by the teardown cluster barrier, which the
    // leader passes only after its bounded MMA drain.
    for (int kt = issued - kPairStages < 0 ? 0 : issued - kPairStages; kt < issued; ++kt) {
      if (!(kt < base_kt && quant)) continue;
      const int s = kt % kPairStages;
      const uint32_t ph = static_cast<uint32_t>(kt / kPairStages) & 1u;
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(smem_u32(&sm.cfull[s]), ph)) {
        if (global_timer_ns() - t0 > p.wait_limit_ns) break;
      }
    }
  }
}

__device__ void pair_mma(const ProjParams& p, const ProjMember& mb, const PairSmem& sm,
                         uint32_t tmem, int base_kt,
                         int total_kt) {
  const bool quant = mb.bits != 0;
  const uint32_t idesc = make_idesc_bf16(2 * kBlockN, static_cast<uint32_t>(p.n_tok));
  uint32_t acc = 0;
  for (int kt = 0; kt < total_kt; ++kt) {
    const int s = kt % kPairStages;
    const uint32_t ph = static_cast<uint32_t>(kt / kPairStages) & 1u;
    if (!mbar_wait(smem_u32(&sm.full[s]), ph, sm.abort, kSiteFull | s, p.wait_limit_ns)) break;
    const bool from_tmem = quant && kt < base_kt;
    if (from_tmem &&
        !mbar_wait(smem_u32(&sm.afull[s]), ph, sm.abort, kSiteDeq | s, p.wait_limit_ns))
      break;
    tc_fence_after();
    MP_TRACE_MARK(kTrMma, kt);
    const uint32_t xaddr = smem_u32(sm.tiles + s * kPairStageBytes);
    const uint32_t waddr = xaddr + kPairXBytes;
#pragma unroll
    for (int kk = 0; kk < kBlockK / 16; ++kk) {
      const uint64_t bdesc = make_sdesc_sw128(xaddr + kk * 32);
      if (from_tmem) {
        umma_ts_pair(tmem + kPairAcc, tmem + kPairACol + s * kPairAStride + kk * 8, bdesc, idesc, acc);
      } else {
        umma_ss_pair(tmem + kPairAcc, make_sdesc_sw128(waddr + kk * 32), bdesc, idesc, acc);
      }
      acc = 1;
    }
    umma_commit_pair(smem_u32(&sm.empty[s]), 0x3);
  }
  if (*sm.abort == 0u) umma_commit_pair(smem_u32(sm.tfull), 0x3);
  umma_commit_pair(smem_u32(sm.drain), 0x1);
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(smem_u32(sm.drain), 0)) {
    if (global_timer_ns() - t0 > p.wait_limit_ns) {
      atomicCAS(const_cast<uint32_t*>(sm.abort), 0u, kSiteDrain);
      break;
    }
  }
}

// Warps 2-9. Warpgroup g converts columns [32g, 32g + 32) of every stage for
// the 128 feature rows of this CTA: thread (warp % 4, lane) owns row r.
__device__ void pair_dequant(const ProjParams& p, const ProjMember& mb, const PairSmem& sm,
                             uint32_t tmem, int f0,
                             int base_kt) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = (warp - 2) >> 2;
  const int q = warp & 3;
  const int r = q * 32 + lane;
  const int n = f0 + r;
  const bool row_ok = n < mb.N;
  const uint32_t* sbrow = mb.sb + static_cast<size_t>(row_ok ? n : 0) * mb.sb_stride;
  const uint32_t taddr0 = (static_cast<uint32_t>(q * 32) << 16) + kPairACol + 16 * g;
  const uint64_t magic2 = f32x2(-mb.code_magic, -mb.code_magic);
  uint4 sbv = make_uint4(0, 0, 0, 0);
  for (int kt = 0; kt < base_kt; ++kt) {
    const int s = kt % kPairStages;
    const uint32_t ph = static_cast<uint32_t>(kt / kPairStages) & 1u;
    if ((kt & 3) == 0) sbv = row_ok ? ld_global_nc_v4(sbrow + kt) : make_uint4(0, 0, 0, 0);
    const uint32_t sbw = pick4p(sbv, kt & 3);
    const float sc = bf16_bits_to_f32(sbw & 0xFFFFu);
    const float bi = bf16_bits_to_f32(sbw >> 16);
    const uint64_t sc2 = f32x2(sc, sc), bi2 = f32x2(bi, bi);
    if (!mbar_wait(smem_u32(&sm.cfull[s]), ph, sm.abort, kSiteCodes | s, p.wait_limit_ns)) break;
    if (threadIdx.x == 64) MP_TRACE_MARK(kTrDeqStart, kt);
    const uint32_t wb = smem_u32(sm.tiles + s * kPairStageBytes + kPairXBytes);
    uint32_t packed[16];
    if (mb.bits == 8) {
      const uint32_t sw = static_cast<uint32_t>((r >> 1) & 3);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint32_t chunk = static_cast<uint32_t>(2 * g + j);
        const uint4 c = ld_shared_v4(wb + r * 64 + ((chunk ^ sw) << 4));
        deq8x4(c.x ^ mb.code_xor, magic2, sc2, bi2, packed[8 * j + 0], packed[8 * j + 1]);
        deq8x4(c.y ^ mb.code_xor, magic2, sc2, bi2, packed[8 * j + 2], packed[8 * j + 3]);
        deq8x4(c.z ^ mb.code_xor, magic2, sc2, bi2, packed[8 * j + 4], packed[8 * j + 5]);
        deq8x4(c.w ^ mb.code_xor, magic2, sc2, bi2, packed[8 * j + 6], packed[8 * j + 7]);
      }
    } else {
      const uint32_t sw = static_cast<uint32_t>((r >> 2) & 1);
      const uint4 c = ld_shared_v4(wb + r * 32 + ((static_cast<uint32_t>(g) ^ sw) << 4));
      deq4x8(c.x, magic2, sc2, bi2, &packed[0]);
      deq4x8(c.y, magic2, sc2, bi2, &packed[4]);
      deq4x8(c.z, magic2, sc2, bi2, &packed[8]);
      deq4x8(c.w, magic2, sc2, bi2, &packed[12]);
    }
    if (threadIdx.x == 64) MP_TRACE_MARK(kTrDeqMath, kt);
    MP_TMEM_ST_32X32B_X16(tmem + taddr0 + s * kPairAStride, packed);
    tmem_wait_st();
    if (threadIdx.x == 64) MP_TRACE_MARK(kTrDeqStored, kt);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&sm.afull[s]), 0));
    if (threadIdx.x == 64) MP_TRACE_MARK(kTrDeqEnd, kt);
  }
}

__device__ __forceinline__ float pair_scale(const EpilogueScale& es, int t, int slot) {
  int g = 0;
  while (g + 1 < es.n_seg && t >= es.seg_start[g + 1]) ++g;
  return es.seg_scale[g][slot];
}

// Warps 2-9: warpgroup g reads token columns [g * n_tok / 2, (g + 1) * n_tok / 2)
// of this CTA's 128 feature rows out of TMEM and rounds them to bf16. Lanes
// pair up (features 2i, 2i+1) with one shuffle per token pair, so each lane
// writes one bf16x2 word of a [n_tok][64]-feature staging half tile laid out
// with the 128-byte swizzle (conflict-free). One thread then stores both
// halves with TMA bulk stores, which clip rows past M and columns past N.
__device__ void pair_epilogue(const ProjParams& p, const ProjMember& mb, const PairSmem& sm,
                              uint32_t tmem, int f0,
                              int t0) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = (warp - 2) >> 2;
  const int q = warp & 3;
  const int fl = q * 32 + lane;  // feature row within this CTA's 128
  const int f = f0 + fl;
  const bool odd = (lane & 1) != 0;
  const bool ok = mbar_wait(smem_u32(sm.tfull), 0, sm.abort, kSiteEpi, p.wait_limit_ns);
  const uint32_t half_bytes = static_cast<uint32_t>(p.n_tok) * 128u;
  if (ok) {
    tc_fence_after();
    if (threadIdx.x == 64) MP_TRACE_MARK(kTrEpiStart, 0);
    int slot = -1;
    if (p.scale.enabled) {
      for (int i = 0; i < p.scale.n_ranges; ++i)
        if (f >= p.scale.range_start[i] && f < p.scale.range_start[i + 1])
          slot = p.scale.range_slot[i];
    }
    const int half = p.n_tok / 2;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    // staging half tile of features [64h, 64h + 64); word (2 features) index in its row
    const uint32_t stage = smem_u32(sm.tiles) + static_cast<uint32_t>(q >> 1) * half_bytes;
    const uint32_t wi = static_cast<uint32_t>(16 * (q & 1) + (lane >> 1));
    const uint32_t chunk = wi >> 2, in_chunk = (wi & 3u) << 2;
    for (int c = 0; c < half / 32; ++c) {
      const int col = g * half + c * 32;
      uint32_t v[32];
      MP_TMEM_LD_32X32B_X32(tmem + lane_base + kPairAcc + col, v);
      tmem_wait_ld();
      if (p.scale.enabled) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float sc = slot >= 0 ? pair_scale(p.scale, t0 + col + j, slot) : 0.0f;
          v[j] = __float_as_uint(__uint_as_float(v[j]) * sc);
        }
      }
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float mine_even = __uint_as_float(v[j]);
        const float mine_odd = __uint_as_float(v[j + 1]);
        const float give = odd ? mine_even : mine_odd;
        const float got = __shfl_xor_sync(0xFFFFFFFFu, give, 1);
        const uint32_t word = odd ? pack_bf16x2(got, mine_odd) : pack_bf16x2(mine_even, got);
        const uint32_t r = static_cast<uint32_t>(col + j + (odd ? 1 : 0));
        const uint32_t addr = stage + r * 128u + (((chunk ^ (r & 7u)) << 4) | in_chunk);
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(word) : "memory");
      }
    }
  }
  // Every epilogue thread passes this barrier (also on the abort path).
  fence_proxy_async_shared();
  named_barrier(1, kDeqThreads);
  if (ok && threadIdx.x == 64 && *sm.abort == 0u) {
    tma_store_2d(&mb.tm_y, smem_u32(sm.tiles), f0, t0);
    tma_store_2d(&mb.tm_y, smem_u32(sm.tiles) + half_bytes, f0 + 64, t0);
    tma_store_commit();
    tma_store_wait_read();
    MP_TRACE_MARK(kTrEpiEnd, 0);
  }
}

}  // namespace

#ifdef MP_TRACE
extern "C" int mp_trace_read(long long* host, int n) {
  const size_t bytes = sizeof(long long) * 2 * kTrEvents * kTraceStages;
  if (n * sizeof(long long) < bytes) return -1;
  return cudaMemcpyFromSymbol(host, g_trace, bytes) == cudaSuccess ? 0 : -2;
}
#endif

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    proj_pair_kernel(const __grid_constant__ ProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  const PairSmem sm = carve_pair(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  int mi = 0;
  while (mi + 1 < p.n_members && pair >= p.mem[mi + 1].pair_begin) ++mi;
  const ProjMember& mb = p.mem[mi];
  const int f0 = (pair - mb.pair_begin) * (2 * kBlockN) + static_cast<int>(rank) * kBlockN;
  const int t0 = blockIdx.y * p.n_tok;
  const int tx0 = t0 + static_cast<int>(rank) * (p.n_tok / 2);
  const int base_kt = (p.K + kBlockK - 1) / kBlockK;  // a ragged last tile (dense only) reads zeros
  const int total_kt = base_kt + mb.lora_ktiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(smem_u32(&sm.full[s]), 1);
      mbar_init(smem_u32(&sm.empty[s]), 1);
      mbar_init(smem_u32(&sm.cfull[s]), 1);
      mbar_init(smem_u32(&sm.afull[s]), 2 * kDeqThreads / 32);  // one arrive per dequant warp
    }
    mbar_init(smem_u32(sm.tfull), 1);
    mbar_init(smem_u32(sm.drain), 1);
    *sm.abort = 0u;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&p.tm_x);
    tma_prefetch_map(&mb.tm_w);
    tma_prefetch_map(&mb.tm_y);
    if (mb.lora_ktiles > 0) {
      tma_prefetch_map(&mb.tm_t);
      tma_prefetch_map(&mb.tm_b);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(sm.tmem_slot), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_slot;

  if (warp == 0) {
    if (lane == 0) pair_producer(p, mb, sm, leader, f0, tx0, base_kt, total_kt);
  } else if (warp == 1) {
    if (lane == 0 && leader) pair_mma(p, mb, sm, tmem, base_kt, total_kt);
  } else {
    if (mb.bits != 0) pair_dequant(p, mb, sm, tmem, f0, base_kt);
    pair_epilogue(p, mb, sm, tmem, f0, t0);
  }

  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
  if (threadIdx.x == 0 && *sm.abort != 0u) atomicOr(p.err, kErrTimeout);
}

// Token rows per pair tile: the widest of 256 / 128 / 64 that still puts at
// least one CTA on every SM, for a launch of `pairs` feature pairs.
int pick_ntok_pair(int m, int pairs) {
  for (int nt : {256, 128}) {
    if (2L * pairs * ((m + nt - 1) / nt) >= 148) return nt;
  }
  return 64;
}

cudaError_t launch_proj_pair(const ProjParams& p, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(proj_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kPairSmemBytes));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid(2 * p.n_pairs, (p.M + p.n_tok - 1) / p.n_tok);
  proj_pair_kernel<<<grid, kPairThreads, kPairSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace mp
