// The fused projection kernel: PERSISTENT CTA pairs (cluster of 2,
// tcgen05 cta_group::2) over a static list of output tiles:
//
//   y[M, N] = x[M, K] · deq(W)[N, K]^T  +  T[M, R] · Bstack[N, R]^T
//
// the reference's `lin` (src/ming-dit.cc:1763-1771) as one pass over K with
// the live LoRA slots appended as extra K tiles. A tile is 256 output features
// x up to 512 tokens; one launch may cover up to four projections of the same
// input (q/k/v, w1/w3), each feature pair mapping to the member whose feature
// range it falls in. Every pair walks the tiles pair_id, pair_id + pairs, ...
//   * each CTA owns 128 of a tile's features (MMA M = 256 across the pair)
//     and loads half of every 256-token sub-tile (MMA N is split across the
//     pair); a 512-token tile keeps two f32 accumulators of 256 TMEM columns,
//     so every dequantized weight stage feeds two MMAs;
//   * warp 0 issues TMA (x sub-tiles and dense / LoRA-B tiles as cta_group::2
//     loads completing on the LEADER's barrier; the codes tile on the CTA's
//     own barrier); warps 2-9 dequantize each CTA's 128 feature rows per
//     64-wide K stage into a bf16 tile in shared memory laid out exactly as a
//     128-byte-swizzled TMA load would lay it out; the leader's warp 1 issues
//     tcgen05.mma.cta_group::2 with both operands in shared memory;
//   * warps 10-13 drain the accumulators of tile i (TMEM -> bf16 -> swizzled
//     staging -> TMA bulk stores) while warps 0-9 already run tile i + 1: the
//     MMAs of tile i + 1 into accumulator j wait only until accumulator j of
//     tile i has been read out.
#include <cuda_runtime.h>

#include "mp_device.cuh"
#include "mp_kernels.h"

namespace mp {

namespace {

constexpr int kMaxStages = 8;          // pipeline stages, at most (per-slot parity bit masks)
constexpr int kSubTok = kMaxTok;       // tokens of one accumulator (MMA N): 256
constexpr uint32_t kABytes = kWStageBytes;            // A: 128 feature rows bf16, 16 KB
constexpr uint32_t kCodesBytes = kBlockN * kBlockK;   // codes: 8-bit at most, 8 KB
constexpr uint32_t kEpiHalfBytes = kEpiRows * 128;    // [64 tokens][64 features] bf16, 8 KB
constexpr uint32_t kEpiBufBytes = 2 * kEpiHalfBytes;  // both feature halves of a CTA
constexpr uint32_t kStagesBytes = 168 * 1024;         // region of the pipeline stages
constexpr uint32_t kTileBytes = kStagesBytes + 2 * kEpiBufBytes;

// Stage s: [x (MMA B operand): this CTA's rows of the tile's token sub-tiles |
// A (MMA A operand: a dense weight or LoRA B tile by TMA, or the dequantized
// codes) | codes]; as many stages as fit in kStagesBytes for the launch's
// token tile NT (3 at 512 tokens, 4 at 256, 5 at 128, 6 at 64: smaller tiles
// finish a stage sooner, so they need more in flight to cover the copy
// latency); then two epilogue staging buffers. Offsets from the
// 1024-byte-aligned tile base. The kernel is instantiated per NT, so the
// stage arithmetic is compile-time.
template <int NT>
struct Geo {
  static constexpr int kSub = NT < kSubTok ? NT : kSubTok;
  static constexpr uint32_t kX = (NT > kSubTok ? 2u : 1u) * (kSub / 2) * 128u;
  static constexpr uint32_t kStage = kX + kABytes + kCodesBytes;
  static constexpr int kStagesFit = static_cast<int>(kStagesBytes / kStage);
  static constexpr int kStages = kStagesFit < kMaxStages ? kStagesFit : kMaxStages;
  static_assert(kStage % 1024u == 0u, "stage alignment");
  __device__ static __forceinline__ uint32_t off_x(int s) { return s * kStage; }
  __device__ static __forceinline__ uint32_t off_a(int s) { return s * kStage + kX; }
  __device__ static __forceinline__ uint32_t off_c(int s) { return s * kStage + kX + kABytes; }
};
__device__ __forceinline__ uint32_t off_epi(int b) { return kStagesBytes + b * kEpiBufBytes; }

// Accumulator orientation. 256- and 512-token tiles keep TOKEN-ROW
// accumulators: TMEM lane = token row (this CTA's half of each 256-token
// sub-tile), column = feature (all 256 of the pair), so an epilogue thread
// holds consecutive features of one token. 64- and 128-token tiles (a
// cta_group::2 MMA with M < 256 puts rows elsewhere in TMEM) keep
// FEATURE-ROW accumulators: lane = feature (this CTA's 128), column = token.
template <int NT>
constexpr bool kTokRows = NT >= kSubTok;
// Token-row epilogue: each warp stages [32 tokens][64 features] (128-byte
// swizzled rows, 4 KB) in one of its two buffers and stores it itself.
constexpr uint32_t kWarpStageBytes = 32 * 128;
static_assert(4 * 2 * kWarpStageBytes == 2 * kEpiBufBytes, "per-warp staging fits the epilogue region");

// warp 0 TMA, warp 1 MMA + TMEM, warps 2-9 dequant, warps 10-13 epilogue
constexpr int kDeqWarp0 = 2;
constexpr int kDeqThreads = 256;
constexpr int kEpiWarp0 = 10;
constexpr int kEpiThreads = 128;
constexpr int kPairThreads = 32 * kEpiWarp0 + kEpiThreads;
constexpr uint32_t kEpiBarrier = 1;  // named barrier of the epilogue warps
// per epilogue warp: the strengths (f32) and slots (int8) of the 256 rank
// columns of a scaled tile
constexpr uint32_t kColBytes = 4 * 256 * (4 + 1);
constexpr uint32_t kPairSmemBytes = kTileBytes + 1024 + 512 + kColBytes;
// attention-head variant only: per epilogue warp, one 16-pair block of the
// rotary tables for its 32 token rows (cos, then sin; rows padded to 80 bytes
// so the row reads are conflict-free)
constexpr uint32_t kRopeRowBytes = 80;
constexpr uint32_t kRopeWarpBytes = 2 * 32 * kRopeRowBytes;
constexpr uint32_t kHeadsSmemBytes = kPairSmemBytes + 4 * kRopeWarpBytes;
static_assert(kHeadsSmemBytes <= 232448, "shared memory per CTA");
static_assert(2 * kSubTok <= kTmemCols, "two accumulators in TMEM");
static_assert(kMaxStages <= 8, "per-slot parity bit masks");

enum : uint32_t {
  kSiteEmpty = 0x1100u,
  kSiteFull = 0x1200u,
  kSiteCodes = 0x1400u,
  kSiteEpi = 0x1500u,
  kSiteDrain = 0x1600u,
  kSiteTmem = 0x1700u,
  kSitePrologue = 0x1800u,
};

// Per-stage timeline of the first CTA pair, only in builds compiled with
// -DMP_TRACE (a profiling build; the product library has no trace code).
#ifdef MP_TRACE
constexpr int kTraceStages = 96;
enum { kTrProducer = 0, kTrDeqStart, kTrDeqEnd, kTrMma, kTrEpiStart, kTrEpiEnd, kTrDeqMath,
       kTrDeqStored, kTrMmaPre, kTrMmaIssued, kTrEvents };
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
  uint64_t* full;    // [stages] leader: both CTAs' TMA tiles and dequantized A tiles of the MMA
  uint64_t* empty;   // [stages] each CTA: stage released by the MMA
  uint64_t* cfull;   // [stages] each CTA: its own codes tile landed
  uint64_t* tfull;   // each CTA: the tile's accumulators complete
  uint64_t* tempty;  // [2] leader: accumulator j read out by both CTAs' epilogues
  uint64_t* drain;   // leader: every MMA issued has completed
  uint32_t* tmem_slot;
  volatile uint32_t* abort;
  float* colscale;   // [4 warps][256] column strengths of a scaled tile
  int8_t* colslot;   // [4 warps][256] column slots (-1: no slot)
  uint8_t* rope;     // [4 warps][kRopeWarpBytes] rotary-table blocks (head variant)
};

__device__ __forceinline__ PairSmem carve_pair(uint8_t* raw) {
  PairSmem s;
  const uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 1023u) & ~uintptr_t(1023u);
  s.tiles = reinterpret_cast<uint8_t*>(base);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s.tiles + kTileBytes);
  s.full = bars;
  s.empty = bars + kMaxStages;
  s.cfull = bars + 2 * kMaxStages;
  s.tfull = bars + 3 * kMaxStages;
  s.tempty = s.tfull + 1;
  s.drain = s.tempty + 2;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.drain + 1);
  s.abort = s.tmem_slot + 1;
  s.colscale = reinterpret_cast<float*>(s.tiles + kTileBytes + 512);
  s.colslot = reinterpret_cast<int8_t*>(s.colscale + 4 * 256);
  s.rope = reinterpret_cast<uint8_t*>(s.colslot + 4 * 256);
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

// One output tile of a launch, as seen by one CTA of the pair.
struct Tile {
  int mi;        // member
  int f0;        // this CTA's first feature row (member-relative)
  int t0;        // first token row
  int z;         // K split
  int n_sub;     // accumulators in use (a second one whose rows all lie past M is dropped)
  int sub;       // tokens per accumulator
  int half;      // token rows of each sub-tile this CTA loads
  int kt_begin;  // K tiles [kt_begin, kt_end); those >= base_kt are appended LoRA tiles
  int kt_end;
};

__device__ __forceinline__ Tile decode_tile(const ProjParams& p, int tile, int rank, int base_kt) {
  Tile t;
  const int per_split = p.n_pairs * p.n_ttiles;
  const int zl = tile / per_split;  // split within this launch
  const int rem = tile - zl * per_split;
  t.z = p.z_first + zl;
  int pair, tt;
  if (p.tile_group <= 1) {
    // token tile fastest: the pairs running at one time share a few feature
    // pairs' weight tiles (each read from memory once, then from L2 by the
    // other token tiles) and sweep the whole of x, which stays in L2 when it
    // fits there
    pair = rem / p.n_ttiles;
    tt = rem - pair * p.n_ttiles;
  } else {
    // groups of tile_group feature pairs, pair fastest within a group: an x
    // tile is read by every pair of the group at about the same time (once
    // from memory when x does not fit in L2), the group's weights stay in L2
    const int per_group = p.tile_group * p.n_ttiles;
    const int g = rem / per_group;
    const int within = rem - g * per_group;
    const int gp = min(p.tile_group, p.n_pairs - g * p.tile_group);
    tt = within / gp;
    pair = g * p.tile_group + (within - tt * gp);
  }
  int mi = 0;
  while (mi + 1 < p.n_members && pair >= p.mem[mi + 1].pair_begin) ++mi;
  t.mi = mi;
  // a SwiGLU pair member covers 128 output features per pair (64 per CTA,
  // each with its W1 and W3 rows), any other member 256 (128 per CTA)
  const int per_cta = p.mem[mi].swiglu ? kBlockN / 2 : kBlockN;
  t.f0 = (pair - p.mem[mi].pair_begin) * (2 * per_cta) + rank * per_cta;
  t.t0 = tt * p.n_tok;
  const int most = p.n_tok > kSubTok ? 2 : 1;
  t.sub = p.n_tok / most;
  t.half = t.sub / 2;
  t.n_sub = (most == 2 && t.t0 + t.sub >= p.M) ? 1 : most;
  t.kt_begin = 0;
  t.kt_end = base_kt + p.mem[mi].lora_ktiles;
  if (p.ksplit > 1) {
    const int base_splits = p.lora_apart ? p.ksplit - 1 : p.ksplit;
    if (t.z >= base_splits) {
      t.kt_begin = base_kt;  // the LoRA split: the appended K tiles only
    } else {
      t.kt_begin = t.z * p.kt_per_split;
      if (t.z + 1 < p.ksplit) t.kt_end = min(base_kt, t.kt_begin + p.kt_per_split);
    }
  }
  return t;
}

// A prologue unit v (fused rank-space pre-GEMM): 256 rank rows x 512 tokens
// of T (two accumulators, as a member tile) over the full K, the stacked A
// as a dense weight.
__device__ __forceinline__ Tile decode_pre(const ProjParams& p, int v, int rank, int base_kt) {
  Tile t;
  const int rp = v % p.pre_rpairs;
  const int tt = v / p.pre_rpairs;
  t.mi = -1;
  t.f0 = rp * (2 * kBlockN) + rank * kBlockN;
  t.t0 = tt * kPreTok;
  t.z = 0;
  t.sub = kSubTok;
  t.half = kSubTok / 2;
  t.n_sub = t.t0 + kSubTok < p.M ? 2 : 1;
  t.kt_begin = 0;
  t.kt_end = base_kt;
  return t;
}

// The units a pair runs, in order: its prologue units, then its member tiles
// p, p + pairs, ... . Prologue units go round-robin to the pairs that run
// the fewest member tiles (those past n_tiles % pairs), filling the idle end
// of the member-tile schedule.
struct UnitIter {
  int pre_next, pre_step, main_next, main_step;
};

__device__ __forceinline__ UnitIter units_begin(const ProjParams& p) {
  const int pairs = static_cast<int>(gridDim.x >> 1);
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int light0 = p.n_tiles % pairs;
  UnitIter u;
  u.main_next = pair;
  u.main_step = pairs;
  u.pre_step = pairs - light0;
  u.pre_next = (p.n_pre > 0 && pair >= light0) ? pair - light0 : p.n_pre;
  return u;
}

// Next unit: -1 - v for prologue unit v, the tile index for a member tile,
// or kNoUnit.
constexpr int kNoUnit = -0x7FFFFFFF;
__device__ __forceinline__ int units_next(const ProjParams& p, UnitIter& u) {
  if (u.pre_next < p.n_pre) {
    const int v = u.pre_next;
    u.pre_next += u.pre_step;
    return -1 - v;
  }
  if (u.main_next < p.n_tiles) {
    const int t = u.main_next;
    u.main_next += u.main_step;
    return t;
  }
  return kNoUnit;
}

__device__ __forceinline__ Tile decode_unit(const ProjParams& p, int unit, int rank, int base_kt) {
  return unit < 0 ? decode_pre(p, -1 - unit, rank, base_kt) : decode_tile(p, unit, rank, base_kt);
}

__device__ __forceinline__ const ProjMember& unit_member(const ProjParams& p, const Tile& t) {
  return t.mi < 0 ? p.pre : p.mem[t.mi];
}

// Fused prologue: bounded wait until every prologue unit holding T rows of
// member tile t has stored them (both CTAs' flags of the needed rank pairs
// and 256-token tiles), then order the coming TMA reads of T after that.
__device__ bool wait_prologue(const ProjParams& p, const ProjMember& mb, const Tile& t,
                              volatile uint32_t* abort) {
  const int rp_lo = mb.t_col / (2 * kBlockN);
  const int rp_hi = (mb.t_col + mb.lora_ktiles * kBlockK - 1) / (2 * kBlockN);
  const int rows_end = min(p.M, t.t0 + t.n_sub * t.sub);
  const int tt_lo = t.t0 / kPreTok;
  const int tt_hi = (rows_end - 1) / kPreTok;
  const uint64_t t0 = global_timer_ns();
  for (int rp = rp_lo; rp <= rp_hi; ++rp) {
    for (int tt = tt_lo; tt <= tt_hi; ++tt) {
      for (int c = 0; c < 2; ++c) {
        const uint32_t* f = p.flags + (static_cast<size_t>(rp) * p.pre_ttiles + tt) * 2 + c;
        while (ld_acquire_gpu(f) != p.epoch) {
          if (*abort != 0u) return false;
          if (global_timer_ns() - t0 > p.wait_limit_ns) {
            atomicCAS(const_cast<uint32_t*>(abort), 0u, kSitePrologue);
            return false;
          }
        }
      }
    }
  }
  fence_proxy_async_global();
  return true;
}

// Warp 0, one thread. Stage iteration `it` runs on across tiles.
template <int NT>
__device__ void pair_producer(const ProjParams& p, const PairSmem& sm, bool leader, int rank,
                              int base_kt) {
  using G = Geo<NT>;
  constexpr uint32_t stages = G::kStages;
  uint32_t it = 0;
  uint32_t cpar = 0;           // per slot: parity of the slot's next codes phase
  uint32_t pend_codes = 0;     // slots whose codes copy this thread has not seen consumed
  uint32_t pend_codes_par = 0;
  uint32_t pend_full = 0;      // slots whose pair copies this thread has not seen consumed
  uint32_t pend_full_par = 0;
  bool aborted = false;
  UnitIter units = units_begin(p);
  for (int unit = units_next(p, units); unit != kNoUnit && !aborted; unit = units_next(p, units)) {
    const Tile t = decode_unit(p, unit, rank, base_kt);
    const ProjMember& mb = unit_member(p, t);
    const bool quant = mb.bits != 0;
    const uint32_t sub_bytes = static_cast<uint32_t>(t.half) * 128u;  // one sub-tile, one CTA
    const uint32_t xbytes_pair = 2u * static_cast<uint32_t>(t.n_sub) * sub_bytes;
    const uint32_t codes_bytes = static_cast<uint32_t>(kBlockN * kBlockK * mb.bits / 8);
    for (int kt = t.kt_begin; kt < t.kt_end; ++kt, ++it) {
      const int s = static_cast<int>(it % stages);
      const uint32_t ph = (it / stages) & 1u;
      const uint32_t bit = 1u << s;
      if (it >= stages &&
          !mbar_wait<true>(smem_u32(&sm.empty[s]), ph ^ 1u, sm.abort, kSiteEmpty | s, p.wait_limit_ns)) {
        aborted = true;
        break;
      }
      pend_codes &= ~bit;  // the MMA consumed the slot's previous copies
      pend_full &= ~bit;
      MP_TRACE_MARK(kTrProducer, static_cast<int>(it));
      const uint32_t xb = smem_u32(sm.tiles) + G::off_x(s);
      const uint32_t wb = smem_u32(sm.tiles) + G::off_a(s);
      const uint32_t full_local = smem_u32(&sm.full[s]);
      const uint32_t full_leader = mapa_shared(full_local, 0);
      const bool lora = kt >= base_kt;
      if (lora && kt == base_kt && p.n_pre > 0 && !wait_prologue(p, mb, t, sm.abort)) {
        aborted = true;
        break;
      }
      const CUtensorMap* xmap = lora ? &mb.tm_t : &p.tm_x;
      const int xk = (lora ? kt - base_kt : kt) * kBlockK;
      if (!lora && quant) {
        if (leader) mbar_arrive_expect_tx(full_local, xbytes_pair);
        const uint32_t cbar = smem_u32(&sm.cfull[s]);
        mbar_arrive_expect_tx(cbar, codes_bytes);
        const int ck = kt * kBlockK * mb.bits / 8;
        if (mb.swiglu) {  // rows 0-63: W1, rows 64-127: W3, both at features f0..f0+63
          tma_load_2d(smem_u32(sm.tiles) + G::off_c(s), &mb.tm_w, cbar, ck, t.f0);
          tma_load_2d(smem_u32(sm.tiles) + G::off_c(s) + codes_bytes / 2, &mb.tm_w3, cbar, ck,
                      t.f0);
        } else {
          tma_load_2d(smem_u32(sm.tiles) + G::off_c(s), &mb.tm_w, cbar, ck, t.f0);
        }
        pend_codes |= bit;
        pend_codes_par = (pend_codes_par & ~bit) | (cpar & bit);
        cpar ^= bit;
      } else {
        if (leader) {
          mbar_arrive_expect_tx(full_local, xbytes_pair + 2u * kWStageBytes);
          mbar_arrive_count(full_local, 2 * kDeqThreads / 32);  // no dequant: the dequantizers' share
        }
        if (lora) {
          // SwiGLU: the interleaved B stack holds 128 rows per 64 features
          tma_load_2d_pair(wb, &mb.tm_b, full_leader, xk, mb.swiglu ? 2 * t.f0 : t.f0);
        } else if (mb.swiglu) {
          tma_load_2d_pair(wb, &mb.tm_w, full_leader, xk, t.f0);
          tma_load_2d_pair(wb + kWStageBytes / 2, &mb.tm_w3, full_leader, xk, t.f0);
        } else {
          tma_load_2d_pair(wb, &mb.tm_w, full_leader, xk, t.f0);
        }
      }
      for (int j = 0; j < t.n_sub; ++j)
        tma_load_2d_pair(xb + j * sub_bytes, xmap, full_leader, xk,
                         t.t0 + j * t.sub + rank * t.half);
      pend_full |= bit;
      pend_full_par = (pend_full_par & ~bit) | ((ph & 1u) << s);
    }
  }
  if (*sm.abort != 0u) {
    // Unwind: wait (bounded) until the copies this CTA still has in flight
    // have landed (the codes on its own barrier; on the leader, both CTAs'
    // pair copies on its full barriers), so none writes shared memory after
    // the CTA has left.
    for (int s = 0; s < static_cast<int>(stages); ++s) {
      const uint32_t bit = 1u << s;
      const uint64_t t0 = global_timer_ns();
      if (pend_codes & bit) {
        while (!mbar_try_wait(smem_u32(&sm.cfull[s]), (pend_codes_par >> s) & 1u))
          if (global_timer_ns() - t0 > p.wait_limit_ns) break;
      }
      if (leader && (pend_full & bit)) {
        while (!mbar_try_wait(smem_u32(&sm.full[s]), (pend_full_par >> s) & 1u))
          if (global_timer_ns() - t0 > p.wait_limit_ns) break;
      }
    }
  }
}

// Warp 1 of the leader, one thread.
template <int NT>
__device__ void pair_mma(const ProjParams& p, const PairSmem& sm, uint32_t tmem, int base_kt) {
  using G = Geo<NT>;
  constexpr uint32_t stages = G::kStages;
  uint32_t it = 0;
  uint32_t tcount = 0;
  bool aborted = false;
  UnitIter units = units_begin(p);
  for (int unit = units_next(p, units); unit != kNoUnit && !aborted;
       unit = units_next(p, units), ++tcount) {
    const Tile t = decode_unit(p, unit, 0, base_kt);
    // token-row tiles: D[token][feature] (A = the x sub-tile, M = its tokens
    // across the pair; B = the weight tile, N = the pair's 256 features);
    // narrower tiles: D[feature][token] (A = weights, B = x)
    const uint32_t idesc =
        kTokRows<NT> ? make_idesc_bf16(static_cast<uint32_t>(t.sub), 2 * kBlockN)
                     : make_idesc_bf16(2 * kBlockN, static_cast<uint32_t>(t.sub));
    const uint32_t acc_cols = kTokRows<NT> ? 2u * kBlockN : static_cast<uint32_t>(t.sub);
    const uint32_t sub_bytes = static_cast<uint32_t>(t.half) * 128u;
    uint32_t acc = 0;
    for (int kt = t.kt_begin; kt < t.kt_end && !aborted; ++kt, ++it) {
      const int s = static_cast<int>(it % stages);
      const uint32_t ph = (it / stages) & 1u;
      MP_TRACE_MARK(kTrMmaPre, static_cast<int>(it));
      if (!mbar_wait<true>(smem_u32(&sm.full[s]), ph, sm.abort, kSiteFull | s, p.wait_limit_ns)) {
        aborted = true;
        break;
      }
      tc_fence_after();
      MP_TRACE_MARK(kTrMma, static_cast<int>(it));
      const uint32_t xaddr = smem_u32(sm.tiles) + G::off_x(s);
      const uint32_t waddr = smem_u32(sm.tiles) + G::off_a(s);
#pragma unroll
      for (int kk = 0; kk < kBlockK / 16; ++kk) {
        const uint64_t wdesc = make_sdesc_sw128(waddr + kk * 32);
        for (int j = 0; j < 2; ++j) {
          if (acc == 0 && tcount > 0) {
            // Accumulator j holds the previous tile until its epilogue has read
            // it out. Both accumulators' phases are waited every tile (also one
            // this tile leaves unused), so no phase is ever skipped.
            if (!mbar_wait<true>(smem_u32(&sm.tempty[j]), (tcount - 1) & 1u, sm.abort, kSiteTmem | j,
                           p.wait_limit_ns)) {
              aborted = true;
              break;
            }
            tc_fence_after();
          }
          if (j >= t.n_sub) continue;
          const uint64_t xdesc = make_sdesc_sw128(xaddr + j * sub_bytes + kk * 32);
          if constexpr (kTokRows<NT>)
            umma_ss_pair(tmem + j * acc_cols, xdesc, wdesc, idesc, acc);
          else
            umma_ss_pair(tmem + j * acc_cols, wdesc, xdesc, idesc, acc);
        }
        if (aborted) break;
        acc = 1;
      }
      if (aborted) break;
      MP_TRACE_MARK(kTrMmaIssued, static_cast<int>(it));
      umma_commit_pair(smem_u32(&sm.empty[s]), 0x3);
    }
    if (!aborted) umma_commit_pair(smem_u32(sm.tfull), 0x3);
  }
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
// the 128 feature rows of this CTA: thread (warp % 4, lane) owns row r. The
// codes tile is 64-byte (w8) or 32-byte (w4) swizzled by its TMA map.
template <int NT>
__device__ void pair_dequant(const ProjParams& p, const PairSmem& sm, int rank, int base_kt) {
  using G = Geo<NT>;
  constexpr uint32_t stages = G::kStages;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = (warp - kDeqWarp0) >> 2;  // K columns [32g, 32g + 32) of every stage
  const int q = warp & 3;
  const int r = q * 32 + lane;
  uint32_t it = 0;
  uint32_t cpar = 0;  // per slot: parity of the slot's next codes phase
  bool aborted = false;
  UnitIter units = units_begin(p);
  for (int unit = units_next(p, units); unit != kNoUnit && !aborted; unit = units_next(p, units)) {
    const Tile t = decode_unit(p, unit, rank, base_kt);
    const ProjMember& mb = unit_member(p, t);
    const int base_end = min(base_kt, t.kt_end);
    if (mb.bits == 0) {  // no dequant stages: keep the stage count in step
      it += static_cast<uint32_t>(t.kt_end - t.kt_begin);
      continue;
    }
    // SwiGLU pair: rows 0-63 are W1's features f0.., rows 64-127 W3's same features
    const int n = mb.swiglu ? t.f0 + (r & 63) : t.f0 + r;
    const bool row_ok = n < mb.N;
    const uint32_t* sbase = (mb.swiglu && r >= 64) ? mb.sb3 : mb.sb;
    const uint32_t* sbrow = sbase + static_cast<size_t>(row_ok ? n : 0) * mb.sb_stride;
    // the row's scale/bias words of 4 groups at a time, the next 4 loaded
    // when the current 4 come into use (a load on the stage that needs it
    // would put a memory round trip on every fourth stage)
    const uint4 zero4 = make_uint4(0, 0, 0, 0);
    uint4 sbv = zero4, sbn = zero4;
    int sb_group = -1;  // which 4 groups sbv holds
    for (int kt = t.kt_begin; kt < base_end; ++kt, ++it) {
      const int s = static_cast<int>(it % stages);
      const int g4 = kt >> 2;
      if (g4 != sb_group) {
        sbv = (sb_group >= 0 && g4 == sb_group + 1) ? sbn
                                                     : (row_ok ? ld_global_nc_v4(sbrow + 4 * g4) : zero4);
        sb_group = g4;
        if (row_ok && 4 * (g4 + 1) < base_end) sbn = ld_global_nc_v4(sbrow + 4 * (g4 + 1));
      }
      const uint32_t sbw = pick4p(sbv, kt & 3);
      const float sc = bf16_bits_to_f32(sbw & 0xFFFFu);
      const float bi = bf16_bits_to_f32(sbw >> 16);
      const float bf = fmaf(-sc, mb.code_offset, bi);
      const uint64_t sc2 = f32x2(sc, sc), bf2 = f32x2(bf, bf);
      if (!mbar_wait<true>(smem_u32(&sm.cfull[s]), (cpar >> s) & 1u, sm.abort, kSiteCodes | s,
                     p.wait_limit_ns)) {
        aborted = true;
        break;
      }
      cpar ^= 1u << s;
      if (threadIdx.x == 64) MP_TRACE_MARK(kTrDeqStart, static_cast<int>(it));
      const uint32_t wb = smem_u32(sm.tiles) + G::off_c(s);
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
      if (threadIdx.x == 64) MP_TRACE_MARK(kTrDeqMath, static_cast<int>(it));
      // Row r of the stage's A tile, K columns [32g, 32g + 32): four 16-byte
      // chunks at the 128-byte-swizzled positions a TMA load would use, then a
      // proxy fence so the tensor core (async proxy) sees the generic stores.
      const uint32_t arow = smem_u32(sm.tiles) + G::off_a(s) + r * 128u;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t chunk =
            (static_cast<uint32_t>(4 * g + c) ^ static_cast<uint32_t>(r & 7)) << 4;
        st_shared_v4(arow + chunk, packed[4 * c], packed[4 * c + 1], packed[4 * c + 2],
                     packed[4 * c + 3]);
      }
      fence_proxy_async_shared();
      if (threadIdx.x == 64) MP_TRACE_MARK(kTrDeqStored, static_cast<int>(it));
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&sm.full[s]), 0));
      if (threadIdx.x == 64) MP_TRACE_MARK(kTrDeqEnd, static_cast<int>(it));
    }
    it += static_cast<uint32_t>(t.kt_end - base_end);  // appended LoRA stages: nothing to do
  }
}

// Row segment of token row t (segments are few; the boundaries are uniform
// across the warp, so these are broadcast parameter loads).
__device__ __forceinline__ int row_segment(const EpilogueScale& es, int t) {
  int g = 0;
  while (g + 1 < es.n_seg && t >= es.seg_start[g + 1]) ++g;
  return g;
}

// Tells the leader's MMA thread that this warp has read accumulator j out.
__device__ __forceinline__ void release_accumulator(const PairSmem& sm, int j) {
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive_remote(mapa_shared(smem_u32(&sm.tempty[j]), 0));
}

// Epilogue variants, one kernel instantiation each (they differ in register
// needs): plain projections, SwiGLU pairs, attention heads.
enum : int { kEpiPlain = 0, kEpiSwiGlu = 1, kEpiHeads = 2 };


// ---- token-row epilogue (256- and 512-token tiles) -------------------------
// Warps 10-13: warp q holds token rows 32q .. 32q + 31 of this CTA's half of a
// sub-tile (TMEM lane quarter q), each thread one token with the pair's 256
// feature columns. Per 64 output features a warp packs its 32 rows into
// bf16x2 words (consecutive features of one token: no shuffles), writes them
// with 16-byte stores into a [32][64] staging box laid out with the 128-byte
// swizzle, and its lane 0 stores the box with one TMA bulk store (which clips
// rows past M and columns past N). Each warp alternates two staging buffers
// of its own, so the warps never wait for one another.

// Before a warp writes a staging buffer: the store that last read it (two
// stores ago) has finished reading.
__device__ __forceinline__ void stage_acquire(int lane) {
  if (lane == 0) tma_store_wait_read_1();
  __syncwarp();
}

// 16 bf16x2 words = features [32h, 32h + 32) of this thread's token row.
__device__ __forceinline__ void stage_words(uint32_t buf, int lane, int h, const uint32_t (&w)[16]) {
  const uint32_t row = buf + static_cast<uint32_t>(lane) * 128u;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t ch = static_cast<uint32_t>(4 * h + i);
    st_shared_v4(row + ((ch ^ static_cast<uint32_t>(lane & 7)) << 4), w[4 * i], w[4 * i + 1],
                 w[4 * i + 2], w[4 * i + 3]);
  }
}

__device__ __forceinline__ void pack_words(const uint32_t (&v)[32], uint32_t (&w)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = pack_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
}

// The warp's staged box: token rows tok0 .. tok0 + 31, output features
// fcol .. fcol + 63 (member-relative; head-major members: head fcol / 128).
__device__ __forceinline__ void stage_store(const ProjMember& mb, uint32_t buf, int fcol, int tok0,
                                            int lane) {
  fence_proxy_async_shared();
  __syncwarp();
  if (lane == 0) {
    if (mb.heads)
      tma_store_3d(&mb.tm_y, buf, fcol % kHeadDim, tok0, fcol / kHeadDim);
    else
      tma_store_2d(&mb.tm_y, buf, fcol, tok0);
    tma_store_commit();
  }
}

// Scaled tiles (rank-space T): the strength of value (token row t, rank
// column c) is seg_scale[segment(t)][slot(c)], 0 outside every slot range.
// Per tile each epilogue warp resolves the slots of the pair's 256 columns
// once (8 per lane) into its shared-memory table; per sub-tile it tabulates
// the strengths for the segment of its first row. Rows of that segment (in
// practice every row: segments are whole images) then read one broadcast
// shared value per column; a warp straddling a segment boundary looks its
// other rows up through the slot table.
__device__ __forceinline__ void column_slots(const EpilogueScale& es, int pf0, int lane,
                                             int8_t* slots) {
#pragma unroll 1
  for (int k = 0; k < 8; ++k) {
    const int c = 32 * k + lane;
    const int col = pf0 + c;
    int slot = -1;
    for (int i = 0; i < es.n_ranges; ++i)
      if (col >= es.range_start[i] && col < es.range_start[i + 1]) slot = es.range_slot[i];
    slots[c] = static_cast<int8_t>(slot);
  }
  __syncwarp();
}

__device__ __forceinline__ void column_scales(const EpilogueScale& es, int g0, int lane,
                                              const int8_t* slots, float* scales) {
  __syncwarp();  // the previous sub-tile's reads of the table are done
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int c = 32 * k + lane;
    const int slot = slots[c];
    scales[c] = slot >= 0 ? es.seg_scale[g0][slot] : 0.0f;
  }
  __syncwarp();
}

// v[jj] *= strength of (this thread's row, column c0 + jj); c0 relative to the pair.
__device__ __forceinline__ void scale_columns(const EpilogueScale& es, bool same_seg, int g, int c0,
                                              const int8_t* slots, const float* scales,
                                              uint32_t (&v)[32]) {
  if (same_seg) {
#pragma unroll
    for (int jj = 0; jj < 32; ++jj)
      v[jj] = __float_as_uint(__uint_as_float(v[jj]) * scales[c0 + jj]);
  } else {
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      const int slot = slots[c0 + jj];
      const float sc = slot >= 0 ? es.seg_scale[g][slot] : 0.0f;
      v[jj] = __float_as_uint(__uint_as_float(v[jj]) * sc);
    }
  }
}

// Plain member (or prologue unit): features pf0 .. pf0 + 255 of the pair.
__device__ void rows_plain(const ProjParams& p, const ProjMember& mb, uint32_t acc, uint32_t stg,
                           int pf0, int tok0, int lane, bool scaled, const int8_t* slots,
                           float* scales, uint32_t& round) {
  int g = 0;
  bool same_seg = true;
  if (scaled) {
    g = row_segment(p.scale, min(tok0 + lane, p.M - 1));
    const int g0 = __shfl_sync(0xFFFFFFFFu, g, 0);
    same_seg = g == g0;
    column_scales(p.scale, g0, lane, slots, scales);
  }
  for (int r = 0; r < 4; ++r) {
    const int fcol = pf0 + 64 * r;
    if (fcol >= mb.N) break;
    const uint32_t buf = stg + (round & 1u) * kWarpStageBytes;
    // both 32-column halves of the box in flight before one wait
    uint32_t v0[32], v1[32];
    MP_TMEM_LD_32X32B_X32(acc + static_cast<uint32_t>(64 * r), v0);
    MP_TMEM_LD_32X32B_X32(acc + static_cast<uint32_t>(64 * r + 32), v1);
    MP_TMEM_WAIT_LD_REGS32(v0);
    MP_TMEM_WAIT_LD_REGS32(v1);
    stage_acquire(lane);
    {
      if (scaled) scale_columns(p.scale, same_seg, g, 64 * r, slots, scales, v0);
      uint32_t w[16];
      pack_words(v0, w);
      stage_words(buf, lane, 0, w);
    }
    {
      if (scaled) scale_columns(p.scale, same_seg, g, 64 * r + 32, slots, scales, v1);
      uint32_t w[16];
      pack_words(v1, w);
      stage_words(buf, lane, 1, w);
    }
    stage_store(mb, buf, fcol, tok0, lane);
    ++round;
  }
}

// Split-K: this thread's token row of the fp32 partial sums, 16-byte stores
// (the rank-space widths split-K runs on are multiples of 64).
__device__ void rows_split(const ProjParams& p, const ProjMember& mb, const Tile& t, uint32_t acc,
                           int pf0, int tok) {
  float* prow = p.part + static_cast<size_t>(t.z) * p.M * p.part_ld + static_cast<size_t>(tok) * p.part_ld;
  for (int r = 0; r < 8; ++r) {
    const int c0 = pf0 + 32 * r;
    if (c0 >= mb.N) break;
    uint32_t v[32];
    MP_TMEM_LD_32X32B_X32(acc + static_cast<uint32_t>(32 * r), v);
    MP_TMEM_WAIT_LD_REGS32(v);
    if (tok < p.M) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (c0 + 4 * i < mb.N)
          *reinterpret_cast<float4*>(prow + c0 + 4 * i) =
              make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                          __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
    }
  }
}

// SwiGLU pair member: the pair's columns are [W1 | W3] of CTA 0's 64 features,
// then [W1 | W3] of CTA 1's, so a thread holds g and u of the same feature:
// h = bf16(g / (1 + exp(-g)) * u) of the bf16 gate and up values, the
// reference's swiglu (src/metal/ming_ops.metal:95-112).
__device__ void rows_swiglu(const ProjMember& mb, uint32_t acc, uint32_t stg, int pf0, int tok0,
                            int lane, uint32_t& round) {
  for (int r = 0; r < 2; ++r) {
    const int fcol = pf0 + 64 * r;
    if (fcol >= mb.N) break;
    const uint32_t buf = stg + (round & 1u) * kWarpStageBytes;
    stage_acquire(lane);
    const uint32_t row = buf + static_cast<uint32_t>(lane) * 128u;
    for (int h = 0; h < 4; ++h) {  // 16 features at a time
      uint32_t gv[16], uv[16];
      MP_TMEM_LD_32X32B_X16(acc + static_cast<uint32_t>(128 * r + 16 * h), gv);
      MP_TMEM_LD_32X32B_X16(acc + static_cast<uint32_t>(128 * r + 64 + 16 * h), uv);
      MP_TMEM_WAIT_LD_REGS16(gv);
      MP_TMEM_WAIT_LD_REGS16(uv);
#pragma unroll
      for (int i4 = 0; i4 < 2; ++i4) {  // one 16-byte chunk (8 features) at a time
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = 8 * i4 + 2 * e;  // features c, c + 1: gate and up rounded as pairs
          const uint32_t gw = pack_bf16x2(__uint_as_float(gv[c]), __uint_as_float(gv[c + 1]));
          const uint32_t uw = pack_bf16x2(__uint_as_float(uv[c]), __uint_as_float(uv[c + 1]));
          const float g[2] = {__uint_as_float(gw << 16), __uint_as_float(gw & 0xFFFF0000u)};
          const float u[2] = {__uint_as_float(uw << 16), __uint_as_float(uw & 0xFFFF0000u)};
          float hv[2];
#pragma unroll
          for (int b = 0; b < 2; ++b) hv[b] = __fdividef(g[b], 1.0f + __expf(-g[b])) * u[b];
          w[e] = pack_bf16x2(hv[0], hv[1]);
        }
        const uint32_t ch = static_cast<uint32_t>(2 * h + i4);
        st_shared_v4(row + ((ch ^ static_cast<uint32_t>(lane & 7)) << 4), w[0], w[1], w[2], w[3]);
      }
    }
    stage_store(mb, buf, fcol, tok0, lane);
    ++round;
  }
}

// Attention-head member: the pair's 256 columns are two heads, stored
// head-major ([heads][M][128], the layout the attention reads; the reference
// transposes into it, src/ming-dit.cc:2085-2088). For q and k (head_norm)
// each token's head row first gets the head's RMSNorm and the rotary
// embedding, with the roundings of the unfused sequence (projection output,
// normed value and rotated value each rounded to bf16; the per-head rms of
// :2083-2084 and tr_rope of :1885-1894):
//   y = bf16(acc);  z = bf16(y * rsqrt(sum(y^2) / 128 + eps) * gain[f])
//   (out[2i], out[2i+1]) = bf16(z[2i] c - z[2i+1] s, z[2i] s + z[2i+1] c)
// with c, s the tables' entries at (token row, i). A first pass over the two
// heads' TMEM columns sums the squares in the thread's own registers
// (features in order). The second pass walks four blocks of 16 rotary pairs
// (32 features of each head); a block of the tables for the warp's 32 rows
// is copied into shared memory with coalesced asynchronous copies (one block
// ahead), and each thread reads its own row from there.

// Block b of the rotary tables (pairs 16b .. 16b + 15) for token rows tok0 ..
// tok0 + 31 into the warp's staging rows: 2 x 32 rows x 64 bytes, four
// 16-byte copies per lane, four lanes per row (rows past M repeat row M - 1).
__device__ __forceinline__ void rope_block_copy(const ProjMember& mb, uint32_t rope, int M, int tok0,
                                                int b, int lane) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int piece = lane + 32 * j;  // 0..127: row piece / 4, 16-byte column piece % 4
    const int row = piece >> 2, col = piece & 3;
    const size_t src = static_cast<size_t>(min(tok0 + row, M - 1)) * (kHeadDim / 2) + 16 * b + 4 * col;
    const uint32_t dst = rope + static_cast<uint32_t>(row) * kRopeRowBytes + 16u * col;
    cp_async_16(dst, mb.rope_cos + src);
    cp_async_16(dst + 32 * kRopeRowBytes, mb.rope_sin + src);
  }
  cp_async_commit();
}

__device__ void rows_heads(const ProjParams& p, const ProjMember& mb, uint32_t acc, uint32_t stg,
                           uint32_t rope, int pf0, int tok0, int lane, uint32_t& round) {
  const bool norm = mb.head_norm != 0;
  const int nh = pf0 + kHeadDim < mb.N ? 2 : 1;  // heads of the pair inside the member
  float rn[2] = {1.0f, 1.0f};
  if (norm) {
    rope_block_copy(mb, rope, p.M, tok0, 0, lane);  // lands during the first pass
    float ss[2] = {0.0f, 0.0f};
    for (int c4 = 0; c4 < 4; ++c4) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        if (hh >= nh) break;
        uint32_t v[32];
        MP_TMEM_LD_32X32B_X32(acc + static_cast<uint32_t>(kHeadDim * hh + 32 * c4), v);
        MP_TMEM_WAIT_LD_REGS32(v);
#pragma unroll
        for (int jj = 0; jj < 32; jj += 2) {
          const uint32_t yw = pack_bf16x2(__uint_as_float(v[jj]), __uint_as_float(v[jj + 1]));
          const float y0 = __uint_as_float(yw << 16), y1 = __uint_as_float(yw & 0xFFFF0000u);
          ss[hh] = __fadd_rn(ss[hh], __fmul_rn(y0, y0));
          ss[hh] = __fadd_rn(ss[hh], __fmul_rn(y1, y1));
        }
      }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
      rn[hh] = rsqrtf(__fadd_rn(__fmul_rn(ss[hh], 1.0f / kHeadDim), mb.norm_eps));
  }
  const uint32_t swz = static_cast<uint32_t>(lane & 7);
  const uint32_t my_row = rope + static_cast<uint32_t>(lane) * kRopeRowBytes;
  for (int b = 0; b < 4; ++b) {  // 16 rotary pairs = features 32b .. 32b + 31 of each head
    const int rr = b >> 1;       // the 64-feature box
    float4 cs[4], sn[4];
    if (norm) {
      cp_async_wait_all();
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        cs[i] = ld_shared_f4(my_row + 16u * i);
        sn[i] = ld_shared_f4(my_row + 32u * kRopeRowBytes + 16u * i);
      }
      __syncwarp();  // every lane has its row: the next block may overwrite
      if (b + 1 < 4) rope_block_copy(mb, rope, p.M, tok0, b + 1, lane);
    }
    if ((b & 1) == 0) {
      // both staging buffers (one box per head): every earlier store has read its buffer
      if (lane == 0) tma_store_wait_read();
      __syncwarp();
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      if (hh >= nh) break;
      const uint32_t row = stg + static_cast<uint32_t>(hh) * kWarpStageBytes +
                           static_cast<uint32_t>(lane) * 128u;
      for (int c2 = 0; c2 < 2; ++c2) {  // 16 features at a time
        const int k = 2 * b + c2;       // 16-feature chunk of the head
        uint32_t v[16];
        MP_TMEM_LD_32X32B_X16(acc + static_cast<uint32_t>(kHeadDim * hh + 16 * k), v);
        MP_TMEM_WAIT_LD_REGS16(v);
        uint32_t w[8];
        if (norm) {
          // the head's gains (the same address in every lane: cached after the first tile)
          const uint4* gp = reinterpret_cast<const uint4*>(mb.norm_w) + 2 * k;
          const uint4 gg[2] = {__ldg(gp), __ldg(gp + 1)};
          const uint64_t rn2 = f32x2(rn[hh], rn[hh]);
#pragma unroll
          for (int i = 0; i < 8; ++i) {  // pair i of the chunk: features 2i, 2i + 1
            const uint4 gq = gg[i >> 2];
            const uint32_t gw = (i & 3) == 0 ? gq.x : (i & 3) == 1 ? gq.y : (i & 3) == 2 ? gq.z : gq.w;
            const int pi = 8 * c2 + i;  // pair within the block
            const float4 cq = cs[pi >> 2], sq = sn[pi >> 2];
            const float c = (pi & 3) == 0 ? cq.x : (pi & 3) == 1 ? cq.y : (pi & 3) == 2 ? cq.z : cq.w;
            const float s = (pi & 3) == 0 ? sq.x : (pi & 3) == 1 ? sq.y : (pi & 3) == 2 ? sq.z : sq.w;
            // packed pairs: y = bf16(acc), z = bf16((y * rn) * gain), then
            // (z0 c, z0 s) + (-(z1 s), z1 c), each product and sum rounded once
            const uint32_t yw = pack_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
            const uint64_t y = f32x2(__uint_as_float(yw << 16), __uint_as_float(yw & 0xFFFF0000u));
            const uint64_t g = f32x2(__uint_as_float(gw << 16), __uint_as_float(gw & 0xFFFF0000u));
            const uint32_t zw = f32x2_to_bf16x2(mul_f32x2(mul_f32x2(y, rn2), g));
            const float z0 = __uint_as_float(zw << 16), z1 = __uint_as_float(zw & 0xFFFF0000u);
            const uint64_t pz = mul_f32x2(f32x2(z0, z0), f32x2(c, s));
            const uint64_t qz = mul_f32x2(f32x2(z1, z1), f32x2(-s, c));
            w[i] = f32x2_to_bf16x2(add_f32x2(pz, qz));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            w[i] = pack_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const uint32_t ch = static_cast<uint32_t>(2 * (k & 3) + e);  // 16-byte chunk of the box row
          st_shared_v4(row + ((ch ^ swz) << 4), w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
        }
      }
    }
    if ((b & 1) == 1) {
      for (int hh = 0; hh < nh; ++hh)
        stage_store(mb, stg + static_cast<uint32_t>(hh) * kWarpStageBytes,
                    pf0 + kHeadDim * hh + 64 * rr, tok0, lane);
    }
  }
  // the warp's next round writes the buffer the NEWEST store did not read
  // (buffer 1 with two heads, buffer 0 with one): its own wait then only has
  // to see the older store done
  round = nh == 2 ? 2u : 1u;
}

template <int EPI>
__device__ void pair_epilogue_rows(const ProjParams& p, const PairSmem& sm, uint32_t tmem, int rank,
                                   int base_kt) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q = warp & 3;
  const bool split = p.part != nullptr;
  const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
  const uint32_t stg = smem_u32(sm.tiles) + kStagesBytes + static_cast<uint32_t>(q) * 2u * kWarpStageBytes;
  int8_t* const slots = sm.colslot + 256 * q;
  float* const scales = sm.colscale + 256 * q;
  uint32_t tcount = 0;
  uint32_t round = 0;
  UnitIter units = units_begin(p);
  for (int unit = units_next(p, units); unit != kNoUnit; unit = units_next(p, units), ++tcount) {
    const Tile t = decode_unit(p, unit, rank, base_kt);
    const ProjMember& mb = unit_member(p, t);
    // strengths apply to a rank-space pre-GEMM launch and to prologue units
    const bool scaled = p.scale.enabled && (p.n_pre == 0 || t.mi < 0);
    const bool ok_mine =
        mbar_wait<true>(smem_u32(sm.tfull), tcount & 1u, sm.abort, kSiteEpi, p.wait_limit_ns);
    if (!named_barrier_and(kEpiBarrier, kEpiThreads, ok_mine)) break;
    tc_fence_after();
    if (threadIdx.x == 32 * kEpiWarp0) MP_TRACE_MARK(kTrEpiStart, static_cast<int>(tcount));
    const bool swiglu = EPI == kEpiSwiGlu && t.mi >= 0 && mb.swiglu;
    const bool heads = EPI == kEpiHeads && t.mi >= 0 && mb.heads;
    const int pf0 = t.f0 - rank * (swiglu ? kBlockN / 2 : kBlockN);  // the pair's first feature
    if (scaled && !split) column_slots(p.scale, pf0, lane, slots);
    for (int j = 0; j < 2; ++j) {
      if (j < t.n_sub) {
        const int tok0 = t.t0 + j * t.sub + rank * t.half + q * 32;  // this warp's first token row
        const uint32_t acc = tmem + lane_base + static_cast<uint32_t>(j * 2 * kBlockN);
        if (tok0 < p.M) {
          if (split)
            rows_split(p, mb, t, acc, pf0, tok0 + lane);
          else if (swiglu)
            rows_swiglu(mb, acc, stg, pf0, tok0, lane, round);
          else if (heads)
            rows_heads(p, mb, acc, stg, smem_u32(sm.rope) + static_cast<uint32_t>(q) * kRopeWarpBytes,
                       pf0, tok0, lane, round);
          else
            rows_plain(p, mb, acc, stg, pf0, tok0, lane, scaled && !split, slots, scales, round);
        }
      }
      release_accumulator(sm, j);
    }
    if (t.mi < 0) {
      // prologue unit: T rows stored (complete, not just read out of shared
      // memory), then published to the member tiles waiting for them
      if (lane == 0) {
        tma_store_wait_all();
        fence_proxy_async_global();
      }
      named_barrier(kEpiBarrier, kEpiThreads);
      if (threadIdx.x == 32 * kEpiWarp0) {
        __threadfence();
        const int v = -1 - unit;
        const int rp = v % p.pre_rpairs, tt = v / p.pre_rpairs;
        st_release_gpu(p.flags + (static_cast<size_t>(rp) * p.pre_ttiles + tt) * 2 + rank, p.epoch);
      }
    }
    if (threadIdx.x == 32 * kEpiWarp0) MP_TRACE_MARK(kTrEpiEnd, static_cast<int>(tcount));
  }
  if (lane == 0) tma_store_wait_all();
}

// ---- feature-row epilogue (64- and 128-token tiles, plain members) ---------
// Warps 10-13 (TMEM lane quarter q = warp % 4: features 32q .. 32q + 31 of the
// CTA's 128). Per accumulator, rounds of 64 tokens: two 32-column TMEM loads,
// lane-pair shuffles into bf16x2 words (features 2i, 2i+1), a [64][64]-feature
// staging half tile per feature half laid out with the 128-byte swizzle, then
// one thread stores both halves with TMA bulk stores (they clip rows past M
// and columns past N). Two staging buffers alternate. In split-K mode the fp32
// sums go straight to the partial-sum array instead.
__device__ void pair_epilogue_cols(const ProjParams& p, const PairSmem& sm, uint32_t tmem,
                                   int rank, int base_kt) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q = warp & 3;
  const int fl = q * 32 + lane;  // feature row within this CTA's 128
  const bool odd = (lane & 1) != 0;
  const bool issuer = threadIdx.x == 32 * kEpiWarp0;
  const bool split = p.part != nullptr;
  const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
  // word (2 features) index within a staging row of 64 features
  const uint32_t wi = static_cast<uint32_t>(16 * (q & 1) + (lane >> 1));
  const uint32_t chunk = wi >> 2, in_chunk = (wi & 3u) << 2;
  uint32_t tcount = 0;
  uint32_t round = 0;
  UnitIter units = units_begin(p);
  for (int unit = units_next(p, units); unit != kNoUnit; unit = units_next(p, units), ++tcount) {
    const Tile t = decode_unit(p, unit, rank, base_kt);
    const ProjMember& mb = unit_member(p, t);
    const int f = t.f0 + fl;
    // strengths apply to a rank-space pre-GEMM launch and to prologue units
    const bool scaled = p.scale.enabled && (p.n_pre == 0 || t.mi < 0);
    const bool ok_mine =
        mbar_wait<true>(smem_u32(sm.tfull), tcount & 1u, sm.abort, kSiteEpi, p.wait_limit_ns);
    if (!named_barrier_and(kEpiBarrier, kEpiThreads, ok_mine)) break;
    tc_fence_after();
    if (threadIdx.x == 32 * kEpiWarp0) MP_TRACE_MARK(kTrEpiStart, static_cast<int>(tcount));
    int slot = -1;
    if (!split && scaled) {
      for (int i = 0; i < p.scale.n_ranges; ++i)
        if (f >= p.scale.range_start[i] && f < p.scale.range_start[i + 1])
          slot = p.scale.range_slot[i];
    }
    for (int j = 0; j < 2; ++j) {
      if (j >= t.n_sub) {
        release_accumulator(sm, j);
        continue;
      }
      // rounds of this accumulator with at least one token row below M (a
      // store box never starts past the output)
      const int rows_left = p.M - (t.t0 + j * t.sub);
      const int rounds = min(t.sub, rows_left) / kEpiRows + (min(t.sub, rows_left) % kEpiRows != 0);
      for (int rr = 0; rr < rounds; ++rr) {
        const int tr0 = t.t0 + j * t.sub + rr * kEpiRows;  // first token row of the round
        if (split) {
          float* prow = p.part + static_cast<size_t>(t.z) * p.M * p.part_ld + f;
          for (int c = 0; c < 2; ++c) {
            uint32_t v[32];
            MP_TMEM_LD_32X32B_X32(
                tmem + lane_base + static_cast<uint32_t>(j * t.sub + rr * kEpiRows + c * 32), v);
            MP_TMEM_WAIT_LD_REGS32(v);
            if (rr + 1 == rounds && c == 1) release_accumulator(sm, j);
            if (f < mb.N) {
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) {
                const int tok = tr0 + c * 32 + jj;
                if (tok < p.M) prow[static_cast<size_t>(tok) * p.part_ld] = __uint_as_float(v[jj]);
              }
            }
          }
          continue;
        }
        const uint32_t buf = smem_u32(sm.tiles) + off_epi(static_cast<int>(round & 1u));
        // the stores that last read this buffer have finished reading (issuer waited)
        named_barrier(kEpiBarrier, kEpiThreads);
        const uint32_t stage = buf + static_cast<uint32_t>(q >> 1) * kEpiHalfBytes;
        for (int c = 0; c < 2; ++c) {
          uint32_t v[32];
          MP_TMEM_LD_32X32B_X32(
              tmem + lane_base + static_cast<uint32_t>(j * t.sub + rr * kEpiRows + c * 32), v);
          MP_TMEM_WAIT_LD_REGS32(v);
          if (rr + 1 == rounds && c == 1) release_accumulator(sm, j);
          if (scaled) {
            // one strength per 32-token chunk unless a row-segment boundary
            // falls inside it (the per-lane slot makes each lookup divergent)
            const int tc = tr0 + c * 32;
            const int g_lo = row_segment(p.scale, tc);
            if (g_lo == row_segment(p.scale, tc + 31)) {
              const float sc = slot >= 0 ? p.scale.seg_scale[g_lo][slot] : 0.0f;
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) v[jj] = __float_as_uint(__uint_as_float(v[jj]) * sc);
            } else {
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) {
                const float sc =
                    slot >= 0 ? p.scale.seg_scale[row_segment(p.scale, tc + jj)][slot] : 0.0f;
                v[jj] = __float_as_uint(__uint_as_float(v[jj]) * sc);
              }
            }
          }
          // The even lane of a pair writes token je, the odd lane token je + 4:
          // rows 4 apart land in opposite halves of the swizzled row, so one
          // store instruction touches 32 distinct banks.
#pragma unroll
          for (int jb = 0; jb < 32; jb += 8) {
#pragma unroll
            for (int d = 0; d < 4; ++d) {
              const int je = jb + d, jo = jb + d + 4;
              const float give = __uint_as_float(odd ? v[je] : v[jo]);
              const float got = __shfl_xor_sync(0xFFFFFFFFu, give, 1);
              const uint32_t word = odd ? pack_bf16x2(got, __uint_as_float(v[jo]))
                                        : pack_bf16x2(__uint_as_float(v[je]), got);
              const uint32_t row = static_cast<uint32_t>(c * 32 + (odd ? jo : je));
              const uint32_t addr = stage + row * 128u + (((chunk ^ (row & 7u)) << 4) | in_chunk);
              asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(word) : "memory");
            }
          }
        }
        fence_proxy_async_shared();
        named_barrier(kEpiBarrier, kEpiThreads);
        if (issuer) {
          tma_store_2d(&mb.tm_y, buf, t.f0, tr0);
          tma_store_2d(&mb.tm_y, buf + kEpiHalfBytes, t.f0 + 64, tr0);
          tma_store_commit();
          tma_store_wait_read_1();  // the other buffer is free again
        }
        ++round;
      }
    }
    if (t.mi < 0 && issuer) {
      // prologue unit: T rows stored (complete, not just read out of shared
      // memory), then published to the member tiles waiting for them
      tma_store_wait_all();
      fence_proxy_async_global();
      __threadfence();
      const int v = -1 - unit;
      const int rp = v % p.pre_rpairs, tt = v / p.pre_rpairs;
      st_release_gpu(p.flags + (static_cast<size_t>(rp) * p.pre_ttiles + tt) * 2 + rank, p.epoch);
    }
    if (threadIdx.x == 32 * kEpiWarp0) MP_TRACE_MARK(kTrEpiEnd, static_cast<int>(tcount));
  }
  if (issuer) tma_store_wait_all();
}

}  // namespace

#ifdef MP_TRACE
extern "C" int mp_trace_read(long long* host, int n) {
  const size_t bytes = sizeof(long long) * 2 * kTrEvents * kTraceStages;
  if (n * sizeof(long long) < bytes) return -1;
  return cudaMemcpyFromSymbol(host, g_trace, bytes) == cudaSuccess ? 0 : -2;
}
#endif

template <int NT, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    proj_pair_kernel(const __grid_constant__ ProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  const PairSmem sm = carve_pair(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const bool leader = rank == 0;
  const int base_kt = (p.K + kBlockK - 1) / kBlockK;  // a ragged last tile (dense only) reads zeros

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMaxStages; ++s) {
      // the leader producer's arrive (with the expected TMA bytes) + one
      // arrive per dequant warp of both CTAs (the producer arrives those
      // itself for stages without dequant work)
      mbar_init(smem_u32(&sm.full[s]), 1 + 2 * kDeqThreads / 32);
      mbar_init(smem_u32(&sm.empty[s]), 1);
      mbar_init(smem_u32(&sm.cfull[s]), 1);
    }
    mbar_init(smem_u32(sm.tfull), 1);
    mbar_init(smem_u32(&sm.tempty[0]), 2 * kEpiThreads / 32);  // one arrive per epilogue warp
    mbar_init(smem_u32(&sm.tempty[1]), 2 * kEpiThreads / 32);
    mbar_init(smem_u32(sm.drain), 1);
    *sm.abort = 0u;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&p.tm_x);
    for (int i = 0; i < p.n_members; ++i) {
      tma_prefetch_map(&p.mem[i].tm_w);
      tma_prefetch_map(&p.mem[i].tm_y);
      if (p.mem[i].lora_ktiles > 0) {
        tma_prefetch_map(&p.mem[i].tm_t);
        tma_prefetch_map(&p.mem[i].tm_b);
      }
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
  // set-up done (shared memory, TMEM, tensor maps): global memory from here on
  pdl_wait();
  pdl_release();

  if (warp == 0) {
    if (lane == 0) pair_producer<NT>(p, sm, leader, rank, base_kt);
  } else if (warp == 1) {
    if (lane == 0 && leader) pair_mma<NT>(p, sm, tmem, base_kt);
  } else if (warp < kEpiWarp0) {
    pair_dequant<NT>(p, sm, rank, base_kt);
  } else {
    if constexpr (kTokRows<NT>)
      pair_epilogue_rows<EPI>(p, sm, tmem, rank, base_kt);
    else
      pair_epilogue_cols(p, sm, tmem, rank, base_kt);
  }

  if (*sm.abort != 0u) {
    // Error path only: let copies issued before the abort land (their
    // completion may be counted on the other CTA's barrier) before either
    // CTA of the pair leaves.
    const uint64_t t_settle = global_timer_ns();
    while (global_timer_ns() - t_settle < 100000ull) __nanosleep(1000);
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
  if (threadIdx.x == 0 && *sm.abort != 0u) atomicOr(p.err, kErrTimeout);
}

int resident_pairs();

// Token rows per pair tile for a launch of `pairs` feature pairs over m rows:
// the tile with the fewest modelled cycles, rounds of resident pairs x cycles
// per 64-wide K stage. A 512-token stage is bound by shared-memory bandwidth
// (~1250 cycles); smaller tiles run more stages in flight and take ~760 /
// ~570 / ~470 cycles at 256 / 128 / 64 tokens. Ties go to the wider tile.
int pick_ntok_pair(int m, int pairs) {
#ifdef MP_FORCE_NTOK
  (void)m;
  (void)pairs;
  return MP_FORCE_NTOK;
#else
  const long long slots = resident_pairs();
  const int tiles[4] = {512, 256, 128, 64};
  const double stage[4] = {1250.0, 760.0, 570.0, 470.0};
  int best = 512;
  double best_cost = 1e300;
  for (int i = 0; i < 4; ++i) {
    const long long units = pairs * static_cast<long long>((m + tiles[i] - 1) / tiles[i]);
    const double cost = static_cast<double>((units + slots - 1) / slots) * stage[i];
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = tiles[i];
    }
  }
  return best;
#endif
}

// Failure-detection self-test: an mbarrier nobody arrives on, waited on with
// the same bounded wait the projection kernel uses; the CTA reports the
// timeout through the context's error word and returns.
__global__ void __launch_bounds__(32) wait_selftest_kernel(uint64_t limit_ns, uint32_t* err) {
  __shared__ uint64_t bar;
  __shared__ uint32_t abort_word;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_word = 0u;
    fence_mbar_init();
  }
  __syncwarp();
  const bool ok = mbar_wait<true>(smem_u32(&bar), 0, &abort_word, 0x1900u, limit_ns);
  __syncwarp();
  if (threadIdx.x == 0 && (!ok || abort_word != 0u)) atomicOr(err, kErrTimeout);
}

cudaError_t launch_wait_selftest(uint64_t limit_ns, uint32_t* err, cudaStream_t stream) {
  wait_selftest_kernel<<<1, 32, 0, stream>>>(limit_ns, err);
  return cudaGetLastError();
}

// Second pass of a split-K launch (ReduceParams). Thread i owns the 4
// consecutive columns (i mod R/4) and walks the rows i / (R/4), + rows_step,
// ...: the column scale slots are looked up once per thread; every row's
// split loads are in flight together and added in split order.
__global__ void __launch_bounds__(256) lora_reduce_kernel(const __grid_constant__ ReduceParams p,
                                                          int rows_step) {
  pdl_wait();
  pdl_release();
  const int cols4 = p.R / 4;
  const int tid = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (tid >= cols4 * rows_step) return;
  const int j = (tid % cols4) * 4;
  int slot[4] = {-1, -1, -1, -1};
  if (p.scale.enabled) {
    for (int i = 0; i < p.scale.n_ranges; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (j + e >= p.scale.range_start[i] && j + e < p.scale.range_start[i + 1])
          slot[e] = p.scale.range_slot[i];
    }
  }
  const size_t split_stride = static_cast<size_t>(p.M) * p.part_ld;
  int g = 0;  // row segment of t (rows only increase)
  for (int t = tid / cols4; t < p.M; t += rows_step) {
    const float* src = p.part + static_cast<size_t>(t) * p.part_ld + j;
    float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int z0 = 0; z0 < p.ksplit; z0 += 8) {  // 8 splits' loads in flight at a time
      float4 part[8];
#pragma unroll
      for (int z = 0; z < 8; ++z)
        if (z0 + z < p.ksplit)
          part[z] = *reinterpret_cast<const float4*>(src + (z0 + z) * split_stride);
#pragma unroll
      for (int z = 0; z < 8; ++z) {
        if (z0 + z < p.ksplit) {
          a.x = (z0 + z == 0) ? part[z].x : a.x + part[z].x;
          a.y = (z0 + z == 0) ? part[z].y : a.y + part[z].y;
          a.z = (z0 + z == 0) ? part[z].z : a.z + part[z].z;
          a.w = (z0 + z == 0) ? part[z].w : a.w + part[z].w;
        }
      }
    }
    float sc[4] = {1.0f, 1.0f, 1.0f, 1.0f};
    if (p.scale.enabled) {
      while (g + 1 < p.scale.n_seg && t >= p.scale.seg_start[g + 1]) ++g;
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[e] = slot[e] >= 0 ? p.scale.seg_scale[g][slot[e]] : 0.0f;
    }
    uint2 w;
    w.x = pack_bf16x2(a.x * sc[0], a.y * sc[1]);
    w.y = pack_bf16x2(a.z * sc[2], a.w * sc[3]);
    *reinterpret_cast<uint2*>(p.out + static_cast<size_t>(t) * p.out_ld + j) = w;
  }
}

cudaError_t launch_lora_reduce(const ReduceParams& p, cudaStream_t stream) {
  // one pass of resident threads (about 1024 per SM) covers rows_step rows
  const int cols4 = p.R / 4;
  int rows_step = (148 * 1024) / cols4;
  if (rows_step > p.M) rows_step = p.M;
  if (rows_step < 1) rows_step = 1;
  const long long threads = static_cast<long long>(cols4) * rows_step;
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, lora_reduce_kernel, p, rows_step);
}

namespace {

bool g_configured[64] = {};
int g_max_pairs[64] = {};

template <int EPI>
constexpr uint32_t smem_bytes() {
  return EPI == kEpiHeads ? kHeadsSmemBytes : kPairSmemBytes;
}

template <int NT, int EPI>
cudaError_t opt_in_smem() {
  return cudaFuncSetAttribute(proj_pair_kernel<NT, EPI>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(smem_bytes<EPI>()));
}

// Opts every instantiation in to its shared memory and finds the CTA pairs
// resident at once (one CTA per SM, the same for every instantiation), which
// the persistent grid fills; once per device.
cudaError_t configure(int* dev_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  *dev_out = dev;
  if (g_configured[dev]) return cudaSuccess;
  for (cudaError_t r : {opt_in_smem<512, kEpiPlain>(), opt_in_smem<256, kEpiPlain>(),
                        opt_in_smem<128, kEpiPlain>(), opt_in_smem<64, kEpiPlain>(),
                        opt_in_smem<512, kEpiSwiGlu>(), opt_in_smem<256, kEpiSwiGlu>(),
                        opt_in_smem<512, kEpiHeads>(), opt_in_smem<256, kEpiHeads>()})
    if (r != cudaSuccess) return r;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = kPairSmemBytes;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, proj_pair_kernel<512, kEpiPlain>, &cfg) !=
          cudaSuccess ||
      clusters <= 0) {
    (void)cudaGetLastError();
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    clusters = sms > 1 ? sms / 2 : 1;
  }
  g_max_pairs[dev] = clusters;
  g_configured[dev] = true;
  return cudaSuccess;
}

template <int NT, int EPI>
cudaError_t launch_nt(const ProjParams& q, int pairs, bool cooperative, cudaStream_t stream) {
  if (cooperative) {
    // Fused prologue: member tiles wait on prologue units of other pairs, so
    // every pair must be resident at once: a cooperative launch of exactly
    // the resident pair count (refused, with nothing run, if it cannot be).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(kPairThreads, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes<EPI>();
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, proj_pair_kernel<NT, EPI>, q);
  }
  // may begin its set-up while the previous launch on the stream finishes
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes<EPI>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, proj_pair_kernel<NT, EPI>, q);
}

}  // namespace

int resident_pairs() {
  int dev = 0;
  if (configure(&dev) != cudaSuccess) return 74;
  return g_max_pairs[dev];
}

cudaError_t launch_proj_pair(const ProjParams& p, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = configure(&dev);
  if (e != cudaSuccess) return e;
  ProjParams q = p;
  q.n_ttiles = (p.M + p.n_tok - 1) / p.n_tok;
  q.n_tiles = q.n_pairs * q.n_ttiles *
              (p.ksplit > 1 ? (p.z_count > 0 ? p.z_count : p.ksplit - p.z_first) : 1);
  const bool coop = q.n_pre > 0;
  if (coop && p.n_tok != kMaxTileTok) return cudaErrorInvalidValue;  // prologue units need NT 512
  const int pairs = coop ? g_max_pairs[dev]
                         : (q.n_tiles < g_max_pairs[dev] ? q.n_tiles : g_max_pairs[dev]);
  bool swiglu = false, heads = false;
  for (int i = 0; i < p.n_members; ++i) {
    swiglu = swiglu || p.mem[i].swiglu != 0;
    heads = heads || p.mem[i].heads != 0;
  }
  if (swiglu && heads) return cudaErrorInvalidValue;
  if (swiglu) {  // SwiGLU pair launches: 512- or 256-token tiles
    switch (p.n_tok) {
      case 512: return launch_nt<512, kEpiSwiGlu>(q, pairs, coop, stream);
      case 256: return launch_nt<256, kEpiSwiGlu>(q, pairs, coop, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  if (heads) {  // attention-head launches: 512- or 256-token tiles
    switch (p.n_tok) {
      case 512: return launch_nt<512, kEpiHeads>(q, pairs, coop, stream);
      case 256: return launch_nt<256, kEpiHeads>(q, pairs, coop, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (p.n_tok) {
    case 512: return launch_nt<512, kEpiPlain>(q, pairs, coop, stream);
    case 256: return launch_nt<256, kEpiPlain>(q, pairs, coop, stream);
    case 128: return launch_nt<128, kEpiPlain>(q, pairs, coop, stream);
    case 64: return launch_nt<64, kEpiPlain>(q, pairs, coop, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mp
