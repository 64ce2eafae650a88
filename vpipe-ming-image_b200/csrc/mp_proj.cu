// The fused projection kernel on CTA PAIRS (cluster of 2, tcgen05 cta_group::2):
//
//   y[M, N] = x[M, K] · deq(W)[N, K]^T  +  T[M, R] · Bstack[N, R]^T
//
// the reference's `lin` (src/ming-dit.cc:1763-1771) as one pass over K with
// the live LoRA slots appended as extra K tiles, on a tile of 256 output
// features x up to 512 tokens per pair of SMs. One launch may cover up to
// four projections of the same input (q/k/v, w1/w3): each pair maps to the
// member whose feature range it falls in.
//   * each CTA owns 128 of the pair's features (MMA M = 256 across the pair)
//     and loads HALF of every 256-token sub-tile (MMA N is split across the
//     pair); a 512-token tile keeps two f32 accumulators of 256 columns in
//     TMEM, so every dequantized weight stage feeds two MMAs;
//   * each CTA dequantizes its own 128 feature rows per 64-wide K stage (two
//     warpgroups, each converting half of the stage's columns with packed
//     f32x2 arithmetic) into a bf16 tile in shared memory laid out exactly as
//     a 128-byte-swizzled TMA load would lay it out, and the leader's single
//     MMA thread issues tcgen05.mma.cta_group::2 with both operands in
//     shared memory;
//   * activation / dense-weight / LoRA tiles complete on the LEADER's full
//     barrier (cta_group::2 TMA); the codes tile of each CTA completes on
//     that CTA's own barrier, where its dequantizers wait; the MMA commit
//     multicasts stage release and accumulator-ready to both CTAs.
#include <cuda_runtime.h>

#include "mp_device.cuh"
#include "mp_kernels.h"

namespace mp {

namespace {

#ifndef MP_PAIR_STAGES
#define MP_PAIR_STAGES 4
#endif
constexpr int kPairStages = MP_PAIR_STAGES;
constexpr int kSubTok = kMaxTok;       // tokens of one accumulator (MMA N): 256
constexpr int kTileTok = kMaxTileTok;  // tokens of a pair tile: two accumulators
constexpr uint32_t kPairXBytes = (kTileTok / 2) * 128;    // x: this CTA's token rows, 32 KB
constexpr uint32_t kPairABytes = kWStageBytes;            // A: 128 feature rows bf16, 16 KB
constexpr uint32_t kPairCodesBytes = kBlockN * kBlockK;   // codes: 8-bit at most, 8 KB
constexpr uint32_t kPairStageBytes = kPairXBytes + kPairABytes + kPairCodesBytes;  // 56 KB

// Stage s: [x (MMA B operand) | A (MMA A operand: a dense weight or LoRA B
// tile by TMA, or the dequantized codes) | codes], from the 1024-byte-aligned
// tile base.
__device__ __forceinline__ uint32_t off_x(int s) { return s * kPairStageBytes; }
__device__ __forceinline__ uint32_t off_a(int s) { return s * kPairStageBytes + kPairXBytes; }
__device__ __forceinline__ uint32_t off_c(int s) {
  return s * kPairStageBytes + kPairXBytes + kPairABytes;
}
constexpr uint32_t kPairTileBytes = kPairStages * kPairStageBytes;

// warp 0 TMA, warp 1 MMA + TMEM, warps 2-9 dequant + epilogue
constexpr int kPairThreads = 320;
constexpr int kDeqThreads = 256;
constexpr uint32_t kPairSmemBytes = kPairTileBytes + 1024 + 512;
static_assert(kPairSmemBytes <= 232448, "shared memory per CTA");
static_assert(kPairTileBytes >= 2 * 2 * kSubTok * 128, "epilogue staging of two accumulators");
static_assert(2 * kSubTok <= kTmemCols, "two accumulators in TMEM");

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
  uint64_t* afull;   // [stages] leader: both CTAs' dequantized A tile written
  uint64_t* tfull;   // each CTA: accumulators complete
  uint64_t* drain;   // leader: every MMA issued has completed
  uint32_t* tmem_slot;
  volatile uint32_t* abort;
};

__device__ __forceinline__ PairSmem carve_pair(uint8_t* raw) {
  PairSmem s;
  const uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 1023u) & ~uintptr_t(1023u);
  s.tiles = reinterpret_cast<uint8_t*>(base);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s.tiles + kPairTileBytes);
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

// Code -> float without a conversion instruction: a byte-permute puts the
// 8-bit code q into bits 8-15 of the float 32768 (bit pattern 0x47000000),
// which is exactly 32768 + q. One packed FMA with the group scale s and the
// folded bias (b - s * code_offset, code_offset = 32768 plus the code's zero
// point) gives s * q + b before the bf16 rounding.
__device__ __forceinline__ float code_as_float(uint32_t w, uint32_t sel) {
  return __uint_as_float(__byte_perm(w, 0x4700u, sel));
}

// 4 packed 8-bit codes -> two bf16x2 words, with packed fp32 pairs.
__device__ __forceinline__ void deq8x4(uint32_t w, uint64_t sc2, uint64_t bf2, uint32_t& p0,
                                       uint32_t& p1) {
  const uint64_t a = f32x2(code_as_float(w, 0x5404u), code_as_float(w, 0x5414u));
  const uint64_t b = f32x2(code_as_float(w, 0x5424u), code_as_float(w, 0x5434u));
  p0 = f32x2_to_bf16x2(fma_f32x2(a, sc2, bf2));
  p1 = f32x2_to_bf16x2(fma_f32x2(b, sc2, bf2));
}

// 8 packed 4-bit codes (code j at bits [4j, 4j+4)) -> four bf16x2 words.
__device__ __forceinline__ void deq4x8(uint32_t w, uint64_t sc2, uint64_t bf2, uint32_t* p) {
  const uint32_t ev = w & 0x0F0F0F0Fu;          // codes 0, 2, 4, 6
  const uint32_t od = (w >> 4) & 0x0F0F0F0Fu;   // codes 1, 3, 5, 7
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t sel = 0x5404u | (static_cast<uint32_t>(b) << 4);
    const uint64_t q = f32x2(code_as_float(ev, sel), code_as_float(od, sel));
    p[b] = f32x2_to_bf16x2(fma_f32x2(q, sc2, bf2));
  }
}

__device__ __forceinline__ uint32_t pick4p(const uint4& v, int i) {
  uint32_t r = v.x;
  r = (i == 1) ? v.y : r;
  r = (i == 2) ? v.z : r;
  r = (i == 3) ? v.w : r;
  return r;
}

// Token geometry of one pair tile at token row t0: `n_sub` accumulators of
// `sub` tokens each (a second accumulator whose rows all lie past M is
// dropped), every CTA holding `half` rows of each sub-tile.
struct TileGeom {
  int n_sub;
  int sub;
  int half;
};

__device__ __forceinline__ TileGeom tile_geom(const ProjParams& p, int t0) {
  TileGeom g;
  const int most = p.n_tok > kSubTok ? 2 : 1;
  g.sub = p.n_tok / most;
  g.half = g.sub / 2;
  g.n_sub = (most == 2 && t0 + g.sub >= p.M) ? 1 : most;
  return g;
}

// K tiles [kt_begin, kt_end): tiles below base_kt are the base weight's,
// the rest are appended LoRA tiles. Stage i of the loop holds tile kt_begin + i.
__device__ void pair_producer(const ProjParams& p, const ProjMember& mb, const PairSmem& sm,
                              const TileGeom& tg, bool leader, int f0, int t0, int rank,
                              int kt_begin, int base_kt, int kt_end) {
  const bool quant = mb.bits != 0;
  const uint32_t sub_bytes = static_cast<uint32_t>(tg.half) * 128u;  // one sub-tile, one CTA
  const uint32_t xbytes_pair = 2u * static_cast<uint32_t>(tg.n_sub) * sub_bytes;
  const uint32_t codes_bytes = static_cast<uint32_t>(kBlockN * kBlockK * mb.bits / 8);
  const int n_kt = kt_end - kt_begin;
  int issued = 0;
  for (int i = 0; i < n_kt; ++i) {
    const int kt = kt_begin + i;
    const int s = i % kPairStages;
    const uint32_t ph = static_cast<uint32_t>(i / kPairStages) & 1u;
    if (i >= kPairStages &&
        !mbar_wait(smem_u32(&sm.empty[s]), ph ^ 1u, sm.abort, kSiteEmpty | s, p.wait_limit_ns))
      break;
    MP_TRACE_MARK(kTrProducer, i);
    const uint32_t xb = smem_u32(sm.tiles) + off_x(s);
    const uint32_t wb = smem_u32(sm.tiles) + off_a(s);
    const uint32_t full_local = smem_u32(&sm.full[s]);
    const uint32_t full_leader = mapa_shared(full_local, 0);
    const bool lora = kt >= base_kt;
    const CUtensorMap* xmap = lora ? &mb.tm_t : &p.tm_x;
    const int xk = (lora ? kt - base_kt : kt) * kBlockK;
    if (!lora && quant) {
      if (leader) mbar_arrive_expect_tx(full_local, xbytes_pair);
      const uint32_t cbar = smem_u32(&sm.cfull[s]);
      mbar_arrive_expect_tx(cbar, codes_bytes);
      tma_load_2d(smem_u32(sm.tiles) + off_c(s), &mb.tm_w, cbar, kt * kBlockK * mb.bits / 8, f0);
    } else {
      if (leader) mbar_arrive_expect_tx(full_local, xbytes_pair + 2u * kWStageBytes);
      tma_load_2d_pair(wb, lora ? &mb.tm_b : &mb.tm_w, full_leader, xk, f0);
    }
    for (int j = 0; j < tg.n_sub; ++j)
      tma_load_2d_pair(xb + j * sub_bytes, xmap, full_leader, xk, t0 + j * tg.sub + rank * tg.half);
    issued = i + 1;
  }
  if (*sm.abort != 0u) {
    // Unwind: wait (bounded) for this CTA's own codes copies still in flight;
    // the pair copies are drained by the teardown cluster barrier, which the
    // leader passes only after its bounded MMA drain.
    for (int i = issued - kPairStages < 0 ? 0 : issued - kPairStages; i < issued; ++i) {
      if (!(kt_begin + i < base_kt && quant)) continue;
      const int s = i % kPairStages;
      const uint32_t ph = static_cast<uint32_t>(i / kPairStages) & 1u;
      const uint64_t t0w = global_timer_ns();
      while (!mbar_try_wait(smem_u32(&sm.cfull[s]), ph)) {
        if (global_timer_ns() - t0w > p.wait_limit_ns) break;
      }
    }
  }
}

__device__ void pair_mma(const ProjParams& p, const ProjMember& mb, const PairSmem& sm,
                         const TileGeom& tg, uint32_t tmem, int kt_begin, int base_kt,
                         int kt_end) {
  const bool quant = mb.bits != 0;
  const uint32_t idesc = make_idesc_bf16(2 * kBlockN, static_cast<uint32_t>(tg.sub));
  const uint32_t sub_bytes = static_cast<uint32_t>(tg.half) * 128u;
  uint32_t acc = 0;
  for (int i = 0; i < kt_end - kt_begin; ++i) {
    const int kt = kt_begin + i;
    const int s = i % kPairStages;
    const uint32_t ph = static_cast<uint32_t>(i / kPairStages) & 1u;
    if (!mbar_wait(smem_u32(&sm.full[s]), ph, sm.abort, kSiteFull | s, p.wait_limit_ns)) break;
    const bool dequantized = quant && kt < base_kt;
    if (dequantized &&
        !mbar_wait(smem_u32(&sm.afull[s]), ph, sm.abort, kSiteDeq | s, p.wait_limit_ns))
      break;
    tc_fence_after();
    MP_TRACE_MARK(kTrMma, i);
    const uint32_t xaddr = smem_u32(sm.tiles) + off_x(s);
    const uint32_t waddr = smem_u32(sm.tiles) + off_a(s);
#pragma unroll
    for (int kk = 0; kk < kBlockK / 16; ++kk) {
      const uint64_t adesc = make_sdesc_sw128(waddr + kk * 32);
      for (int j = 0; j < tg.n_sub; ++j) {
        const uint64_t bdesc = make_sdesc_sw128(xaddr + j * sub_bytes + kk * 32);
        umma_ss_pair(tmem + static_cast<uint32_t>(j * tg.sub), adesc, bdesc, idesc, acc);
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
// The codes tile is 64-byte (w8) or 32-byte (w4) swizzled by its TMA map.
__device__ void pair_dequant(const ProjParams& p, const ProjMember& mb, const PairSmem& sm,
                             int f0, int kt_begin, int base_end) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = (warp - 2) >> 2;  // K columns [32g, 32g + 32) of every stage
  const int q = warp & 3;
  const int r = q * 32 + lane;
  const int n = f0 + r;
  const bool row_ok = n < mb.N;
  const uint32_t* sbrow = mb.sb + static_cast<size_t>(row_ok ? n : 0) * mb.sb_stride;
  uint4 sbv = make_uint4(0, 0, 0, 0);
  int sb_group = -1;  // which 4 groups sbv holds
  for (int i = 0; i < base_end - kt_begin; ++i) {
    const int kt = kt_begin + i;
    const int s = i % kPairStages;
    const uint32_t ph = static_cast<uint32_t>(i / kPairStages) & 1u;
    if ((kt >> 2) != sb_group) {
      sbv = row_ok ? ld_global_nc_v4(sbrow + (kt & ~3)) : make_uint4(0, 0, 0, 0);
      sb_group = kt >> 2;
    }
    const uint32_t sbw = pick4p(sbv, kt & 3);
    const float sc = bf16_bits_to_f32(sbw & 0xFFFFu);
    const float bi = bf16_bits_to_f32(sbw >> 16);
    const float bf = fmaf(-sc, mb.code_offset, bi);
    const uint64_t sc2 = f32x2(sc, sc), bf2 = f32x2(bf, bf);
    if (!mbar_wait(smem_u32(&sm.cfull[s]), ph, sm.abort, kSiteCodes | s, p.wait_limit_ns)) break;
    if (threadIdx.x == 64) MP_TRACE_MARK(kTrDeqStart, i);
    const uint32_t wb = smem_u32(sm.tiles) + off_c(s);
    uint32_t packed[16];
    if (mb.bits == 8) {
      const uint32_t sw = static_cast<uint32_t>((r >> 1) & 3);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint32_t chunk = static_cast<uint32_t>(2 * g + j);
        const uint4 c = ld_shared_v4(wb + r * 64 + ((chunk ^ sw) << 4));
        deq8x4(c.x ^ mb.code_xor, sc2, bf2, packed[8 * j + 0], packed[8 * j + 1]);
        deq8x4(c.y ^ mb.code_xor, sc2, bf2, packed[8 * j + 2], packed[8 * j + 3]);
        deq8x4(c.z ^ mb.code_xor, sc2, bf2, packed[8 * j + 4], packed[8 * j + 5]);
        deq8x4(c.w ^ mb.code_xor, sc2, bf2, packed[8 * j + 6], packed[8 * j + 7]);
      }
    } else {
      const uint32_t sw = static_cast<uint32_t>((r >> 2) & 1);
      const uint4 c = ld_shared_v4(wb + r * 32 + ((static_cast<uint32_t>(g) ^ sw) << 4));
      deq4x8(c.x, sc2, bf2, &packed[0]);
      deq4x8(c.y, sc2, bf2, &packed[4]);
      deq4x8(c.z, sc2, bf2, &packed[8]);
      deq4x8(c.w, sc2, bf2, &packed[12]);
    }
    if (threadIdx.x == 64) MP_TRACE_MARK(kTrDeqMath, i);
    // Row r of the stage's A tile, K columns [32g, 32g + 32): four 16-byte
    // chunks at the 128-byte-swizzled positions a TMA load would use, then a
    // proxy fence so the tensor core (async proxy) sees the generic stores.
    const uint32_t arow = smem_u32(sm.tiles) + off_a(s) + r * 128u;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t chunk = (static_cast<uint32_t>(4 * g + c) ^ static_cast<uint32_t>(r & 7)) << 4;
      st_shared_v4(arow + chunk, packed[4 * c], packed[4 * c + 1], packed[4 * c + 2],
                   packed[4 * c + 3]);
    }
    fence_proxy_async_shared();
    if (threadIdx.x == 64) MP_TRACE_MARK(kTrDeqStored, i);
    __syncwarp();
    if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&sm.afull[s]), 0));
    if (threadIdx.x == 64) MP_TRACE_MARK(kTrDeqEnd, i);
  }
}

__device__ __forceinline__ float pair_scale(const EpilogueScale& es, int t, int slot) {
  int g = 0;
  while (g + 1 < es.n_seg && t >= es.seg_start[g + 1]) ++g;
  return es.seg_scale[g][slot];
}

// Warps 2-9: for each accumulator j, warpgroup g reads token columns
// [g * sub / 2, (g + 1) * sub / 2) of this CTA's 128 feature rows out of TMEM
// and rounds them to bf16. Lanes pair up (features 2i, 2i+1) with one shuffle
// per token pair, so each lane writes one bf16x2 word of a [sub][64]-feature
// staging half tile laid out with the 128-byte swizzle (conflict-free). One
// thread then stores the halves with TMA bulk stores, which clip rows past M
// and columns past N. In split-K mode the fp32 sums go straight to the
// partial-sum array instead.
__device__ void pair_epilogue(const ProjParams& p, const ProjMember& mb, const PairSmem& sm,
                              const TileGeom& tg, uint32_t tmem, int f0, int t0) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = (warp - 2) >> 2;
  const int q = warp & 3;
  const int fl = q * 32 + lane;  // feature row within this CTA's 128
  const int f = f0 + fl;
  const bool odd = (lane & 1) != 0;
  const bool ok = mbar_wait(smem_u32(sm.tfull), 0, sm.abort, kSiteEpi, p.wait_limit_ns);
  const uint32_t half_bytes = static_cast<uint32_t>(tg.sub) * 128u;  // one staging half tile
  const bool split = p.part != nullptr;
  const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
  const int cols = tg.sub / 2;  // per warpgroup and accumulator
  if (ok) {
    tc_fence_after();
    if (threadIdx.x == 64) MP_TRACE_MARK(kTrEpiStart, 0);
  }
  if (ok && split) {
    // Lanes own consecutive features, so every warp store is 128 contiguous bytes.
    float* prow = p.part + static_cast<size_t>(blockIdx.z) * p.M * p.part_ld + f;
    for (int j = 0; j < tg.n_sub; ++j) {
      for (int c = 0; c < cols / 32; ++c) {
        const int col = g * cols + c * 32;
        uint32_t v[32];
        MP_TMEM_LD_32X32B_X32(tmem + lane_base + static_cast<uint32_t>(j * tg.sub + col), v);
        MP_TMEM_WAIT_LD_REGS32(v);
        if (f < mb.N) {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int t = t0 + j * tg.sub + col + jj;
            if (t < p.M) prow[static_cast<size_t>(t) * p.part_ld] = __uint_as_float(v[jj]);
          }
        }
      }
    }
  } else if (ok) {
    int slot = -1;
    if (p.scale.enabled) {
      for (int i = 0; i < p.scale.n_ranges; ++i)
        if (f >= p.scale.range_start[i] && f < p.scale.range_start[i + 1])
          slot = p.scale.range_slot[i];
    }
    // word (2 features) index within a staging row of 64 features
    const uint32_t wi = static_cast<uint32_t>(16 * (q & 1) + (lane >> 1));
    const uint32_t chunk = wi >> 2, in_chunk = (wi & 3u) << 2;
    // Chunks of 32 token columns, in (accumulator, column) order.
    const int nck = cols / 32;
    const int total = tg.n_sub * nck;
    auto col_of = [&](int i) { return (i / nck) * tg.sub + g * cols + (i % nck) * 32; };
    auto convert = [&](int i, uint32_t(&v)[32]) {
      const int j = i / nck;
      const int col = g * cols + (i % nck) * 32;  // within accumulator j
      // staging half tile of features [64h, 64h + 64) of accumulator j
      const uint32_t stage =
          smem_u32(sm.tiles) + static_cast<uint32_t>(2 * j + (q >> 1)) * half_bytes;
      if (p.scale.enabled) {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const float sc =
              slot >= 0 ? pair_scale(p.scale, t0 + j * tg.sub + col + jj, slot) : 0.0f;
          v[jj] = __float_as_uint(__uint_as_float(v[jj]) * sc);
        }
      }
#pragma unroll
      for (int jj = 0; jj < 32; jj += 2) {
        const float mine_even = __uint_as_float(v[jj]);
        const float mine_odd = __uint_as_float(v[jj + 1]);
        const float give = odd ? mine_even : mine_odd;
        const float got = __shfl_xor_sync(0xFFFFFFFFu, give, 1);
        const uint32_t word = odd ? pack_bf16x2(got, mine_odd) : pack_bf16x2(mine_even, got);
        const uint32_t r = static_cast<uint32_t>(col + jj + (odd ? 1 : 0));
        const uint32_t addr = stage + r * 128u + (((chunk ^ (r & 7u)) << 4) | in_chunk);
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(word) : "memory");
      }
    };
    for (int i = 0; i < total; ++i) {
      uint32_t v[32];
      MP_TMEM_LD_32X32B_X32(tmem + lane_base + static_cast<uint32_t>(col_of(i)), v);
      MP_TMEM_WAIT_LD_REGS32(v);
      convert(i, v);
    }
  }
  // Every epilogue thread passes this barrier (also on the abort path).
  fence_proxy_async_shared();
  named_barrier(1, kDeqThreads);
  if (ok && !split && threadIdx.x == 64 && *sm.abort == 0u) {
    for (int j = 0; j < tg.n_sub; ++j) {
      const uint32_t st = smem_u32(sm.tiles) + static_cast<uint32_t>(2 * j) * half_bytes;
      tma_store_2d(&mb.tm_y, st, f0, t0 + j * tg.sub);
      tma_store_2d(&mb.tm_y, st + half_bytes, f0 + 64, t0 + j * tg.sub);
    }
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
  const TileGeom tg = tile_geom(p, t0);
  const int base_kt = (p.K + kBlockK - 1) / kBlockK;  // a ragged last tile (dense only) reads zeros
  int kt_begin = 0, kt_end = base_kt + mb.lora_ktiles;
  if (p.ksplit > 1) {
    kt_begin = static_cast<int>(blockIdx.z) * p.kt_per_split;
    if (static_cast<int>(blockIdx.z) + 1 < p.ksplit) kt_end = min(base_kt, kt_begin + p.kt_per_split);
  }
  const int base_end = min(base_kt, kt_end);

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
    if (lane == 0)
      pair_producer(p, mb, sm, tg, leader, f0, t0, static_cast<int>(rank), kt_begin, base_kt,
                    kt_end);
  } else if (warp == 1) {
    if (lane == 0 && leader) pair_mma(p, mb, sm, tg, tmem, kt_begin, base_kt, kt_end);
  } else {
    if (mb.bits != 0) pair_dequant(p, mb, sm, f0, kt_begin, base_end);
    pair_epilogue(p, mb, sm, tg, tmem, f0, t0);
  }

  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
  if (threadIdx.x == 0 && *sm.abort != 0u) atomicOr(p.err, kErrTimeout);
}

// Token rows per pair tile for a launch of `pairs` feature pairs over m rows:
// 512 (two accumulators: every dequantized stage feeds two MMAs) unless 256
// finishes in fewer modelled waves, where a 512-row tile counts as 0.85 of two
// 256-row tiles; below one full wave of 256-row tiles, the widest of 128 / 64
// that still puts a CTA on every SM.
int pick_ntok_pair(int m, int pairs) {
#ifdef MP_FORCE_NTOK
  (void)m;
  (void)pairs;
  return MP_FORCE_NTOK;
#else
  const long long slots = 74;  // pairs resident at once: one CTA per SM
  auto waves = [&](int nt) { return (pairs * static_cast<long long>((m + nt - 1) / nt) + slots - 1) / slots; };
  if (pairs * static_cast<long long>((m + 255) / 256) >= slots) {
    return 0.85 * 2.0 * static_cast<double>(waves(512)) <= static_cast<double>(waves(256)) ? 512 : 256;
  }
  if (pairs * static_cast<long long>((m + 127) / 128) >= slots) return 128;
  return 64;
#endif
}

// Second pass of a split-K launch (ReduceParams): one thread per 4
// consecutive columns of one token row; the splits are added in z order.
__global__ void __launch_bounds__(256) lora_reduce_kernel(const __grid_constant__ ReduceParams p) {
  const int cols4 = p.R / 4;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int t = static_cast<int>(idx / cols4);
  if (t >= p.M) return;
  const int j = static_cast<int>(idx % cols4) * 4;
  const size_t split_stride = static_cast<size_t>(p.M) * p.part_ld;
  const float* src = p.part + static_cast<size_t>(t) * p.part_ld + j;
  // all splits' loads in flight at once, then the sum in split order
  float4 part[kMaxSplits];
#pragma unroll
  for (int z = 0; z < kMaxSplits; ++z)
    if (z < p.ksplit) part[z] = *reinterpret_cast<const float4*>(src + z * split_stride);
  float4 a = part[0];
#pragma unroll
  for (int z = 1; z < kMaxSplits; ++z) {
    if (z < p.ksplit) {
      a.x += part[z].x;
      a.y += part[z].y;
      a.z += part[z].z;
      a.w += part[z].w;
    }
  }
  float sc[4] = {1.0f, 1.0f, 1.0f, 1.0f};
  if (p.scale.enabled) {
    int g = 0;
    while (g + 1 < p.scale.n_seg && t >= p.scale.seg_start[g + 1]) ++g;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int slot = -1;
      for (int i = 0; i < p.scale.n_ranges; ++i)
        if (j + e >= p.scale.range_start[i] && j + e < p.scale.range_start[i + 1])
          slot = p.scale.range_slot[i];
      sc[e] = slot >= 0 ? p.scale.seg_scale[g][slot] : 0.0f;
    }
  }
  uint2 w;
  w.x = pack_bf16x2(a.x * sc[0], a.y * sc[1]);
  w.y = pack_bf16x2(a.z * sc[2], a.w * sc[3]);
  *reinterpret_cast<uint2*>(p.out + static_cast<size_t>(t) * p.out_ld + j) = w;
}

cudaError_t launch_lora_reduce(const ReduceParams& p, cudaStream_t stream) {
  const long long threads = static_cast<long long>(p.M) * (p.R / 4);
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  lora_reduce_kernel<<<blocks, 256, 0, stream>>>(p);
  return cudaGetLastError();
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
  dim3 grid(2 * p.n_pairs, (p.M + p.n_tok - 1) / p.n_tok, p.ksplit > 1 ? p.ksplit : 1);
  proj_pair_kernel<<<grid, kPairThreads, kPairSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace mp
