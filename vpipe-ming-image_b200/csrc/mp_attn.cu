// Non-causal attention with head dim 128 on tcgen05, the consumer of the
// projections' head-major q / k / v: for head h and query row i,
//
//   o[i, 128h .. 128h + 127] = softmax(scale · q_i · K^T) · V
//
// the reference's run_attn over the joint rows of a block (src/ming-dit.cc:
// 1905-2039; q, k and v as its tr_rope / transpose leave them). A CTA PAIR
// (cluster of 2, cta_group::2 MMAs with M = 256) takes 256 query rows of one
// head, 128 per CTA; each step covers 128 keys:
//   * per step each CTA loads only its half of the operands the pair MMA
//     splits along N: 64 keys of K_j (for S = Q · K^T, N = keys) and 64 head
//     dims of V_j (for O += P · V, N = head dims); K / V traffic per FLOP is
//     half that of single-CTA tiles. Warp 0 loads Q once and the K ring
//     (4 stages), warp 10 the V ring (4 stages); every pair load completes on
//     the leader CTA's barrier. The MMA thread commits once per step, after
//     P_j · V_j and S_{j+2} (which the tensor core completes in issue order),
//     to barrier (j + 2) % 4 of one ring: its phase says S_{j+2} is ready for
//     the softmax, K stage (j + 2) % 4 and V stage j % 4 are free for the
//     producers, and O includes P_j · V_j;
//   * each CTA's softmax warps copy its Q rows into TMEM once; warp 1 of the
//     leader then issues S_j = Q · K_j^T with Q read from TMEM (so the only
//     shared-memory operand is the K half) into S[j % 2] of both CTAs, two
//     tiles ahead of O += P_j · V_j, which reads P from TMEM (written over
//     S[j % 2] by the softmax) and V as an MN-major operand straight from its
//     [keys][dims] tile;
//   * warps 2-9 of each CTA (thread = query row, TMEM lane; two warps per row,
//     one per 64-key half of each tile) read S_j into registers once
//     and write P_j = 2^(s·c − m) in bf16
//     (c = scale·log2 e) over its half of S_j's columns with the row sum, in
//     packed f32x2 arithmetic, three of every eight exponential pairs on the
//     FMA pipe and the rest on the MUFU. The exponent base m is the row
//     maximum seen when it was last raised: only when a tile's maximum
//     exceeds it by more than 8 (a factor 256) does the warp rescale its rows
//     of O in TMEM (after the previous P·V has landed) and move m up;
//     otherwise p <= 256 and O, the row sum and the final quotient stay exact
//     relative to the older m;
//   * after the last step the rows of O are divided by their sums and stored
//     bf16 token-major.
// S_{j+1}, S_{j+2} and P_{j-1} · V_{j-1} run while the softmax of tile j
// works (S is double-buffered). The kernel is persistent: each CTA pair
// walks the (head, 256-row block) tiles cid, cid + pairs, ... and its rings,
// barrier phases and S buffers run on as one stream of steps across tiles,
// so the next tile's Q and first K / V tiles load, and its first two S tiles
// are computed, while the softmax warps finish the previous tile (its Q is
// copied into TMEM as soon as the previous tile's last S has completed; the
// output is read out of TMEM before the next tile's first P · V overwrites
// it). Keys past S are masked (their tiles read
// zeros); rows past S are computed and not stored. No TMA multicast. Every
// wait is bounded; on a timeout the CTA unwinds and reports MP_ETIMEOUT.
#include <cuda_runtime.h>

#include <algorithm>

#include "mp_device.cuh"
#include "mp_kernels.h"

namespace mp {

namespace {

constexpr int kAttnTile = 128;                          // query rows per CTA, keys per step
constexpr uint32_t kQBlk = 128 * 64 * 2;                // Q: [128 rows][64 dims] bf16, one TMA box
constexpr uint32_t kQBytes = 2 * kQBlk;                 // Q: 128 rows x 128 dims
constexpr uint32_t kKBlk = 64 * 64 * 2;                 // K half: [64 keys][64 dims], one TMA box
constexpr uint32_t kKHalf = 2 * kKBlk;                  // this CTA's 64 keys x 128 dims
constexpr uint32_t kVHalf = 128 * 64 * 2;               // this CTA's 64 dims of 128 keys, one box
constexpr int kKStages = 4;
constexpr int kVStages = 4;
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kQBytes;             // K ring
constexpr uint32_t kOffV = kOffK + kKStages * kKHalf;   // V ring
constexpr uint32_t kAttnTiles = kOffV + kVStages * kVHalf;  // 160 KB
// row maxima [step parity][half][row], then the row sums of a tile's end [half][row]
constexpr uint32_t kXchgBytes = 3 * 2 * 128 * 4;
static_assert(kKStages == kVStages, "one completion ring for the K and V stages");
static_assert((2 + 3 * kKStages + 4) * 8 + 8 <= 256, "barrier region");
constexpr uint32_t kAttnSmem = kAttnTiles + 1024 + 256 + kXchgBytes;
static_assert(kAttnSmem <= 232448, "shared memory per CTA");
constexpr int kAttnThreads = 352;  // warp 0 Q+K, 1 MMA, 2-9 softmax, 10 V
constexpr int kSoftWarps = 8;      // two per TMEM lane quarter: keys 0-63 / 64-127 of each row
static_assert(kAttnTiles % 1024 == 0, "barrier region after the tiles");
constexpr uint32_t kAttnCols = 512;  // Q (64), S[0] S[1] (128 each), O (128)
constexpr uint32_t kColQ = 0;        // Q rows as bf16 pairs (the A operand of S = Q · K^T)
constexpr uint32_t kColS = 64;       // S[b] (f32) at 64 + 128 b; P_j (bf16 pairs) overwrites S[j % 2]
constexpr uint32_t kColO = 320;      // the O accumulator (f32)
constexpr float kRescaleLog2 = 8.0f;                    // move m only when a max exceeds it by this

enum : uint32_t { kAttnSiteWait = 0x2100u, kAttnSiteDrain = 0x2200u };

struct AttnSmem {
  uint8_t* tiles;
  uint64_t* q_full;
  uint64_t* q_empty;  // every softmax warp of this CTA has copied the tile's Q rows to TMEM
  uint64_t* k_full;   // [kKStages]
  uint64_t* v_full;   // [kVStages]
  uint64_t* q_ready;  // leader: every softmax warp of the pair has put its Q part in TMEM
  uint64_t* done;     // [kKStages] phase i / 4 of barrier i % 4: S_i and P_{i-2} · V_{i-2}
                      // complete in both CTAs (for i >= n only the latter)
  uint64_t* p_full;   // [2] leader: P_j written over S_j by every softmax warp of the pair
  uint64_t* drain;
  uint32_t* tmem_slot;
  volatile uint32_t* abort;
  float* xchg;        // [2][2][128] partial row maxima (then the partial row sums)
};

__device__ __forceinline__ AttnSmem carve_attn(uint8_t* raw) {
  AttnSmem s;
  const uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 1023u) & ~uintptr_t(1023u);
  s.tiles = reinterpret_cast<uint8_t*>(base);
  uint64_t* b = reinterpret_cast<uint64_t*>(s.tiles + kAttnTiles);
  s.q_full = b;
  s.q_empty = s.q_full + 1;
  s.k_full = s.q_empty + 1;
  s.v_full = s.k_full + kKStages;
  s.q_ready = s.v_full + kVStages;
  s.done = s.q_ready + 1;
  s.p_full = s.done + kKStages;
  s.drain = s.p_full + 2;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.drain + 1);
  s.abort = s.tmem_slot + 1;
  s.xchg = reinterpret_cast<float*>(s.tiles + kAttnTiles + 256);
  return s;
}

// K-major operand of `rows` rows x 128 dims as two [rows][64] 128-byte-
// swizzled blocks of `blk` bytes: the 16-wide K step kk sits in block kk / 4
// at byte 32 (kk % 4).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile, uint32_t blk, int kk) {
  return make_sdesc_sw128(tile + static_cast<uint32_t>(kk >> 2) * blk +
                          static_cast<uint32_t>(kk & 3) * 32u);
}

// This CTA's half of V as the MN-major B operand of P · V: [128 keys][64
// dims], one 128-byte-swizzled block (8-key x 64-dim swizzle atoms of 1024
// bytes, one atom wide along N). A 16-key step starts 2048 bytes further;
// 8-key groups are 1024 bytes apart (SBO); the leading byte offset (the next
// 64-dim block) is not reached by a 64-wide half.
__device__ __forceinline__ uint64_t vmn_desc(uint32_t tile, int kk) {
  uint64_t d = 0;
  const uint32_t a = tile + static_cast<uint32_t>(kk) * 2048u;
  d |= static_cast<uint64_t>((a & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(kVHalf >> 4) << 16;    // leading byte offset (unused: one block)
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

// 2^x for a packed pair on the FMA pipe (offloads the MUFU): the Cody-Waite
// split x = i + f with i = round(x) (the 1.5 * 2^23 rounding constant) and
// f in [-0.5, 0.5], a cubic for 2^f (coefficients fitted for this kernel by
// minimizing the maximum relative error on [-0.5, 0.5]: 7.5e-5, far below the
// bf16 rounding of P), and 2^i added to the exponent bits. x is clamped at
// -126 (2^-126 stands in for smaller values; masked keys never get here).
__device__ __forceinline__ uint64_t ex2_poly2(float x0, float x1) {
  const uint64_t x = f32x2(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
  const uint64_t magic = f32x2(12582912.0f, 12582912.0f);
  const uint64_t t = add_f32x2(x, magic);
  const uint64_t r = add_f32x2(t, f32x2(-12582912.0f, -12582912.0f));
  const uint64_t f = fma_f32x2(r, f32x2(-1.0f, -1.0f), x);  // x - r, exact
  uint64_t q = fma_f32x2(f32x2(0.05517144f, 0.05517144f), f, f32x2(0.24261071f, 0.24261071f));
  q = fma_f32x2(q, f, f32x2(0.69326097f, 0.69326097f));
  q = fma_f32x2(q, f, f32x2(0.99992812f, 0.99992812f));
  const uint32_t lo = static_cast<uint32_t>(q) + (static_cast<uint32_t>(t) << 23);
  const uint32_t hi = static_cast<uint32_t>(q >> 32) + (static_cast<uint32_t>(t >> 32) << 23);
  return (static_cast<uint64_t>(hi) << 32) | lo;
}

__device__ __forceinline__ bool attn_wait(const AttnSmem& sm, uint64_t* bar, uint32_t parity,
                                          uint64_t limit) {
  return mbar_wait(smem_u32(bar), parity, sm.abort, kAttnSiteWait, limit);
}

// The tiles of this CTA pair: (head, 256-row block) tile cid + t * ncl for
// t < tiles (cid = the pair's index, ncl = pairs in the grid), n steps each.
struct AttnSched {
  int cid, ncl, nq, n, tiles;
};

__device__ __forceinline__ AttnSched attn_sched(const AttnParams& p) {
  AttnSched s;
  s.n = (p.S + kAttnTile - 1) / kAttnTile;
  s.nq = (p.S + 2 * kAttnTile - 1) / (2 * kAttnTile);
  const int total = s.nq * p.NH;
  s.cid = static_cast<int>(blockIdx.x >> 1);
  s.ncl = static_cast<int>(gridDim.x >> 1);
  s.tiles = s.cid < total ? (total - s.cid + s.ncl - 1) / s.ncl : 0;
  return s;
}

// Head and this CTA's first query row of the pair's tile t.
__device__ __forceinline__ void attn_tile(const AttnSched& s, int t, int rank, int& q0, int& head) {
  const int tile = s.cid + t * s.ncl;
  head = tile / s.nq;
  q0 = (tile - head * s.nq) * 2 * kAttnTile + rank * kAttnTile;
}

// Warp 0 of each CTA, one thread: per tile its Q rows, then its halves of
// the K ring (pair loads completing on the leader's barriers; the leader
// expects both CTAs' bytes). g counts steps over all of the pair's tiles.
__device__ void attn_producer_k(const AttnParams& p, const AttnSmem& sm, const AttnSched& sc,
                                bool leader, int rank) {
  const uint32_t base = smem_u32(sm.tiles);
  int g = 0;
  for (int t = 0; t < sc.tiles; ++t) {
    int q0, head;
    attn_tile(sc, t, rank, q0, head);
    // this CTA's Q rows, on its own barrier (its softmax warps copy them to
    // TMEM), once the previous tile's Q has left shared memory
    if (t > 0 && !attn_wait(sm, sm.q_empty, static_cast<uint32_t>(t - 1) & 1u, p.wait_limit_ns))
      return;
    mbar_arrive_expect_tx(smem_u32(sm.q_full), kQBytes);
    tma_load_3d(base + kOffQ, &p.tm_q, smem_u32(sm.q_full), 0, q0, head);
    tma_load_3d(base + kOffQ + kQBlk, &p.tm_q, smem_u32(sm.q_full), 64, q0, head);
    for (int j = 0; j < sc.n; ++j, ++g) {
      const int st = g % kKStages;
      // K_{g - 4} is free once S_{g - 4} has completed
      if (g >= kKStages &&
          !attn_wait(sm, &sm.done[st], static_cast<uint32_t>(g / kKStages - 1) & 1u,
                     p.wait_limit_ns))
        return;
      const uint32_t kb = base + kOffK + static_cast<uint32_t>(st) * kKHalf;
      const uint32_t bar = mapa_shared(smem_u32(&sm.k_full[st]), 0);
      if (leader) mbar_arrive_expect_tx(smem_u32(&sm.k_full[st]), 2 * kKHalf);
      const int key0 = j * kAttnTile + rank * 64;
      tma_load_3d_pair(kb, &p.tm_k, bar, 0, key0, head);
      tma_load_3d_pair(kb + kKBlk, &p.tm_k, bar, 64, key0, head);
    }
  }
}

// Warp 10 of each CTA, one thread: its 64 dims of the V ring.
__device__ void attn_producer_v(const AttnParams& p, const AttnSmem& sm, const AttnSched& sc,
                                bool leader, int rank) {
  const uint32_t base = smem_u32(sm.tiles);
  int g = 0;
  for (int t = 0; t < sc.tiles; ++t) {
    int q0, head;
    attn_tile(sc, t, rank, q0, head);
    for (int j = 0; j < sc.n; ++j, ++g) {
      const int st = g % kVStages;
      // V_{g - 4} is free once P_{g - 4} · V has completed: barrier i = g - 2
      if (g >= kVStages &&
          !attn_wait(sm, &sm.done[(g - 2) % kKStages],
                     static_cast<uint32_t>((g - 2) / kKStages) & 1u, p.wait_limit_ns))
        return;
      const uint32_t vb = base + kOffV + static_cast<uint32_t>(st) * kVHalf;
      const uint32_t bar = mapa_shared(smem_u32(&sm.v_full[st]), 0);
      if (leader) mbar_arrive_expect_tx(smem_u32(&sm.v_full[st]), 2 * kVHalf);
      tma_load_3d_pair(vb, &p.tm_v, bar, rank * 64, j * kAttnTile, head);
    }
  }
}

// Warp 1 of the leader, one thread: pair MMAs for both CTAs, over the steps
// g of all the pair's tiles (tile g / n, key tile g % n).
__device__ void attn_mma(const AttnParams& p, const AttnSmem& sm, const AttnSched& sc,
                         uint32_t tmem) {
  const uint32_t base = smem_u32(sm.tiles);
  const uint32_t idesc_qk = make_idesc_bf16(2 * kAttnTile, kAttnTile);  // M 256, N 128
  const uint32_t idesc_pv = idesc_qk | (1u << 16);  // B (V) MN-major
  const int n = sc.n;
  const int steps = sc.tiles * n;
  // tile and step within it of the next S and the next P · V, kept as
  // counters (no division on the issue path)
  int s_tile = 0, s_j = 0, pv_j = 0;
  auto issue_s = [&](int g) -> bool {
    // a tile's first S waits for its Q rows in both CTAs' TMEM
    if (s_j == 0 &&
        !attn_wait(sm, sm.q_ready, static_cast<uint32_t>(s_tile) & 1u, p.wait_limit_ns))
      return false;
    if (++s_j == n) {
      s_j = 0;
      ++s_tile;
    }
    const int st = g % kKStages;
    if (!attn_wait(sm, &sm.k_full[st], static_cast<uint32_t>(g / kKStages) & 1u, p.wait_limit_ns))
      return false;
    tc_fence_after();
    const uint32_t kt = base + kOffK + static_cast<uint32_t>(st) * kKHalf;
    // S[g % 2] held P_{g-2}, which P_{g-2} · V (issued before this) reads
    // first: the tensor core runs a thread's MMAs in order
    const uint32_t sc_col = tmem + kColS + 128u * static_cast<uint32_t>(g & 1);
    // A = Q from each CTA's TMEM: 16 dims (8 columns of bf16 pairs) per step
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      umma_ts_pair(sc_col, tmem + kColQ + static_cast<uint32_t>(kk) * 8u,
                   kmajor_desc(kt, kKBlk, kk), idesc_qk, kk > 0 ? 1u : 0u);
    umma_commit_pair(smem_u32(&sm.done[st]), 0x3);  // with P_{g-2} · V before it
    return true;
  };
  auto issue_pv = [&](int g) -> bool {
    const int b = g & 1;
    const int st = g % kVStages;
    if (!attn_wait(sm, &sm.v_full[st], static_cast<uint32_t>(g / kVStages) & 1u, p.wait_limit_ns))
      return false;
    if (!attn_wait(sm, &sm.p_full[b], static_cast<uint32_t>(g >> 1) & 1u, p.wait_limit_ns))
      return false;
    tc_fence_after();
    const uint32_t vt = base + kOffV + static_cast<uint32_t>(st) * kVHalf;
    // A = P_g from each CTA's TMEM, over S[b]: keys 64h .. 64h + 63 as bf16
    // pairs in columns 64h .. 64h + 31 of the buffer; 16 keys per step. A
    // tile's first P · V overwrites O (read out by then: the softmax warps
    // store the previous tile's output before they write this P).
    const bool first = pv_j == 0;
    if (++pv_j == n) pv_j = 0;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      umma_ts_pair(tmem + kColO,
                   tmem + kColS + 128u * static_cast<uint32_t>(b) +
                       64u * static_cast<uint32_t>(kk >> 2) + 8u * static_cast<uint32_t>(kk & 3),
                   vmn_desc(vt, kk), idesc_pv, (!first || kk > 0) ? 1u : 0u);
    return true;  // committed with S_{g+2} (or alone past the last S)
  };
  // S runs two steps ahead of P · V: S_{g+2} is computed while the softmax
  // works on S_{g+1}, so the tensor core never waits for the softmax to have
  // read a tile before the next one can start
  bool ok = true;
  if (steps > 0) ok = issue_s(0);
  if (ok && steps > 1) ok = issue_s(1);
  for (int g = 0; ok && g < steps; ++g) {
    ok = issue_pv(g);
    if (ok && g + 2 < steps)
      ok = issue_s(g + 2);
    else if (ok)
      umma_commit_pair(smem_u32(&sm.done[(g + 2) % kKStages]), 0x3);
  }
  // every MMA issued has completed before TMEM is freed
  umma_commit_pair(smem_u32(sm.drain), 0x1);
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(smem_u32(sm.drain), 0)) {
    if (global_timer_ns() - t0 > p.wait_limit_ns) {
      atomicCAS(const_cast<uint32_t*>(sm.abort), 0u, kAttnSiteDrain);
      break;
    }
  }
}

// A softmax thread's Q row of tile t, dims [64 half, 64 half + 64), from the
// 128-byte-swizzled smem tile into TMEM as bf16 pairs (column = dim / 2);
// then shared memory is free for the next tile's Q and the leader's MMA
// thread may issue the tile's S.
__device__ __forceinline__ bool attn_copy_q(const AttnParams& p, const AttnSmem& sm, uint32_t tmem,
                                            int t, int half, int row, uint32_t lane_base) {
  const bool w = attn_wait(sm, sm.q_full, static_cast<uint32_t>(t) & 1u, p.wait_limit_ns);
  if (!__all_sync(0xFFFFFFFFu, w)) return false;
  const uint32_t qrow = smem_u32(sm.tiles) + kOffQ + static_cast<uint32_t>(half) * kQBlk +
                        static_cast<uint32_t>(row) * 128u;
  uint32_t qv[32];
#pragma unroll
  for (int ch = 0; ch < 8; ++ch) {
    const uint32_t a = qrow + ((static_cast<uint32_t>(ch) ^ static_cast<uint32_t>(row & 7)) << 4);
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(qv[4 * ch]), "=r"(qv[4 * ch + 1]), "=r"(qv[4 * ch + 2]), "=r"(qv[4 * ch + 3])
                 : "r"(a));
  }
  MP_TMEM_ST_32X32B_X32(tmem + lane_base + kColQ + 32u * half, qv);
  tmem_wait_st();
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    mbar_arrive(smem_u32(sm.q_empty));
    mbar_arrive_remote(mapa_shared(smem_u32(sm.q_ready), 0));
  }
  return true;
}

// Warps 2-9: two warps per TMEM lane quarter; thread = query row (lane),
// half = which 64 keys of each 128-key tile (and which 64 columns of O) this
// warp takes. The two halves of a row exchange their partial maxima through
// shared memory (one named barrier per quarter pair and step) and so move
// the row's exponent base identically; each keeps its own partial row sum,
// added to the other once at the tile's end.
__device__ void attn_softmax(const AttnParams& p, const AttnSmem& sm, const AttnSched& sc,
                             uint32_t tmem, int rank) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int quarter = warp & 3;
  const int half = (warp - 2) >> 2;
  const int row = quarter * 32 + lane;
  const uint32_t bar_id = 1u + static_cast<uint32_t>(quarter);  // the quarter's two warps
  const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
  const float c = p.scale_log2;
  const uint64_t c2 = f32x2(c, c);
  // schedule values recomputed from the parameters where used (fewer live
  // registers through the steps)
  const int n = (p.S + kAttnTile - 1) / kAttnTile;
  if (sc.tiles == 0 || !attn_copy_q(p, sm, tmem, 0, half, row, lane_base)) return;
  int g = 0;  // steps over all of the pair's tiles
  for (int t = 0; t < attn_sched(p).tiles; ++t) {
  float m_used = -INFINITY, l = 0.0f;
  for (int j = 0; j < n; ++j, ++g) {
    const int b = g & 1;
    bool w = attn_wait(sm, &sm.done[g % kKStages], static_cast<uint32_t>(g / kKStages) & 1u,
                       p.wait_limit_ns);
    if (!__all_sync(0xFFFFFFFFu, w)) return;
    tc_fence_after();
    const uint32_t sb = tmem + lane_base + kColS + 128u * static_cast<uint32_t>(b) + 64u * half;
    uint32_t sv[64];
    uint32_t* const s1 = sv + 32;
    MP_TMEM_LD_32X32B_X32(sb, sv);
    MP_TMEM_LD_32X32B_X32(sb + 32u, s1);
    MP_TMEM_WAIT_LD_REGS32(sv);
    MP_TMEM_WAIT_LD_REGS32(s1);
    const int valid = p.S - j * kAttnTile - 64 * half;  // keys of this half below S (may be <= 0)
    const bool full = valid >= 64;  // the same in every thread of the warp
    float mx;
    if (full) {
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < 64; i += 8) {
#pragma unroll
        for (int a = 0; a < 4; ++a)
          m4[a] = max3_f32(m4[a], __uint_as_float(sv[i + 2 * a]), __uint_as_float(sv[i + 2 * a + 1]));
      }
      mx = max3_f32(m4[0], m4[1], fmaxf(m4[2], m4[3]));
    } else {
      mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; ++i)
        if (i < valid) mx = fmaxf(mx, __uint_as_float(sv[i]));
    }
    // the row's maximum over both halves
    float* xm = sm.xchg + b * 256;
    xm[half * 128 + row] = mx;
    named_barrier(bar_id, 64);
    mx = fmaxf(mx, xm[(1 - half) * 128 + row]);
    const float mc = mx * c;
    if (j == 0) {
      m_used = mc;
    } else {
      const bool need = mc > m_used + kRescaleLog2;
      if (__any_sync(0xFFFFFFFFu, need)) {
        // O holds P_0..P_{j-1} · V relative to m_used: once P_{j-1} · V has
        // landed (with S_{g+1}: barrier g + 1), scale this warp's half of its
        // rows to the new base
        w = attn_wait(sm, &sm.done[(g + 1) % kKStages],
                      static_cast<uint32_t>((g + 1) / kKStages) & 1u, p.wait_limit_ns);
        if (!__all_sync(0xFFFFFFFFu, w)) return;
        tc_fence_after();
        const float alpha = need ? ex2(m_used - mc) : 1.0f;
#pragma unroll
        for (int c2i = 0; c2i < 2; ++c2i) {
          uint32_t ov[32];
          const uint32_t oa = tmem + lane_base + kColO + 64u * half + static_cast<uint32_t>(32 * c2i);
          MP_TMEM_LD_32X32B_X32(oa, ov);
          MP_TMEM_WAIT_LD_REGS32(ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          MP_TMEM_ST_32X32B_X32(oa, ov);
        }
        tmem_wait_st();
        l *= alpha;
        if (need) m_used = mc;
      }
    }
    float sum = 0.0f;
    uint64_t acc2[2] = {0ull, 0ull};  // packed partial row sums (full halves)
    const uint64_t nm2 = f32x2(-m_used, -m_used);
    // P_j over this warp's own (already read) half of S[b]
    const uint32_t pcol = sb;
#pragma unroll
    for (int c4 = 0; c4 < 2; ++c4) {
      uint32_t w16[16];
      if (full) {
        // 3 of every 8 pairs on the FMA pipe, the rest on the MUFU
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int key = 32 * c4 + 2 * i;
          const uint64_t a = fma_f32x2(f32x2(__uint_as_float(sv[key]), __uint_as_float(sv[key + 1])),
                                       c2, nm2);
          uint64_t e;
          if ((i & 7) < 3)
            e = ex2_poly2(f32x2_lo(a), f32x2_hi(a));
          else
            e = f32x2(ex2(f32x2_lo(a)), ex2(f32x2_hi(a)));
          acc2[i & 1] = add_f32x2(acc2[i & 1], e);
          w16[i] = f32x2_to_bf16x2(e);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int key = 32 * c4 + 2 * i;
          const float p0 = key < valid ? ex2(fmaf(__uint_as_float(sv[key]), c, -m_used)) : 0.0f;
          const float p1 =
              key + 1 < valid ? ex2(fmaf(__uint_as_float(sv[key + 1]), c, -m_used)) : 0.0f;
          sum += p0 + p1;
          w16[i] = pack_bf16x2(p0, p1);
        }
      }
      MP_TMEM_ST_32X32B_X16(pcol + static_cast<uint32_t>(16 * c4), w16);
    }
    if (full) {
      const uint64_t t2 = add_f32x2(acc2[0], acc2[1]);
      sum = f32x2_lo(t2) + f32x2_hi(t2);
    }
    l += sum;
    tmem_wait_st();     // P_j (and an O rescale) written to TMEM
    tc_fence_before();  // ... before P_j · V is issued
    __syncwarp();
    if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&sm.p_full[b]), 0));
  }
  // the tile's last S has completed (waited above): the next tile's Q may
  // replace this one in TMEM
  if (t + 1 < attn_sched(p).tiles && !attn_copy_q(p, sm, tmem, t + 1, half, row, lane_base))
    return;
  // all of O: the tile's last P · V (step g - 1) landed, with S_{g+1}:
  // barrier g + 1
  {
    const bool w = attn_wait(sm, &sm.done[(g + 1) % kKStages],
                             static_cast<uint32_t>((g + 1) / kKStages) & 1u, p.wait_limit_ns);
    if (!__all_sync(0xFFFFFFFFu, w)) return;
    tc_fence_after();
  }
  // the row sum over both halves (added in half order), in a buffer of its
  // own: the next tile's first maxima go to buffer g % 2 while the partner
  // warp may still read this
  float* xl = sm.xchg + 2 * 256;
  xl[half * 128 + row] = l;
  named_barrier(bar_id, 64);
  const float lt = xl[row] + xl[128 + row];
  int q0, head;
  attn_tile(attn_sched(p), t, rank, q0, head);
  const int q = q0 + row;
  const float inv = 1.0f / lt;
  uint16_t* dst = p.o + static_cast<size_t>(q) * p.ldo + static_cast<size_t>(head) * 128 + 64 * half;
#pragma unroll
  for (int c4 = 0; c4 < 2; ++c4) {
    uint32_t ov[32];
    MP_TMEM_LD_32X32B_X32(tmem + lane_base + kColO + 64u * half + static_cast<uint32_t>(32 * c4), ov);
    MP_TMEM_WAIT_LD_REGS32(ov);
    if (q < p.S) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 wv;
        wv.x = pack_bf16x2(__uint_as_float(ov[8 * i]) * inv, __uint_as_float(ov[8 * i + 1]) * inv);
        wv.y = pack_bf16x2(__uint_as_float(ov[8 * i + 2]) * inv, __uint_as_float(ov[8 * i + 3]) * inv);
        wv.z = pack_bf16x2(__uint_as_float(ov[8 * i + 4]) * inv, __uint_as_float(ov[8 * i + 5]) * inv);
        wv.w = pack_bf16x2(__uint_as_float(ov[8 * i + 6]) * inv, __uint_as_float(ov[8 * i + 7]) * inv);
        *reinterpret_cast<uint4*>(dst + 32 * c4 + 8 * i) = wv;
      }
    }
  }
  }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kAttnThreads, 1)
    attn_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  const AttnSmem sm = carve_attn(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const bool leader = rank == 0;
  const AttnSched sc = attn_sched(p);
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(sm.q_full), 1);
    mbar_init(smem_u32(sm.q_empty), kSoftWarps);  // this CTA's softmax warps
    for (int st = 0; st < kKStages; ++st) {
      mbar_init(smem_u32(&sm.k_full[st]), 1);
      mbar_init(smem_u32(&sm.v_full[st]), 1);
      mbar_init(smem_u32(&sm.done[st]), 1);
    }
    mbar_init(smem_u32(sm.q_ready), 2 * kSoftWarps);  // leader: every softmax warp of the pair
    for (int b = 0; b < 2; ++b) mbar_init(smem_u32(&sm.p_full[b]), 2 * kSoftWarps);
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
    tmem_alloc_pair(smem_u32(sm.tmem_slot), kAttnCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_slot;
  if (warp == 0) {
    if (lane == 0) attn_producer_k(p, sm, sc, leader, rank);
  } else if (warp == 1) {
    if (lane == 0 && leader) attn_mma(p, sm, sc, tmem);
  } else if (warp == 10) {
    if (lane == 0) attn_producer_v(p, sm, sc, leader, rank);
  } else {
    attn_softmax(p, sm, sc, tmem, rank);
  }
  if (*sm.abort != 0u) {
    // error path only: let copies issued before the abort land before leaving
    const uint64_t t_settle = global_timer_ns();
    while (global_timer_ns() - t_settle < 100000ull) __nanosleep(1000);
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kAttnCols);
  if (threadIdx.x == 0 && *sm.abort != 0u) atomicOr(p.err, kErrTimeout);
}

bool g_attn_configured[64] = {};
int g_attn_pairs[64] = {};  // CTA pairs of this kernel resident at once

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
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(kAttnThreads, 1, 1);
    cfg.dynamicSmemBytes = kAttnSmem;
    int pairs = 0;
    if (cudaOccupancyMaxActiveClusters(&pairs, attn_kernel, &cfg) != cudaSuccess || pairs <= 0) {
      (void)cudaGetLastError();
      int sms = 0;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      pairs = sms > 1 ? sms / 2 : 1;
    }
    g_attn_pairs[dev] = pairs;
    g_attn_configured[dev] = true;
  }
  // persistent CTA pairs, at most one per (head, 256-row block) tile. With a
  // single 128-key step per tile (S <= 128) every tile gets a pair of its
  // own: a pair's step stream commits a tile's last P · V together with the
  // S two steps later, which would then belong to a tile whose Q can only
  // arrive after this tile's output is stored.
  const long long tiles = static_cast<long long>((p.S + 2 * kAttnTile - 1) / (2 * kAttnTile)) * p.NH;
  const long long pairs = p.S > kAttnTile ? std::min<long long>(tiles, g_attn_pairs[dev]) : tiles;
  if (pairs <= 0 || pairs > (1ll << 30)) return cudaErrorInvalidValue;
  attn_kernel<<<dim3(static_cast<unsigned>(2 * pairs), 1, 1), kAttnThreads, kAttnSmem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace mp
