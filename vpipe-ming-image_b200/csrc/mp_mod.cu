// Batched adaLN modulation for all modulated blocks in ONE launch (per <= 8
// tokens).
//
// The reference runs `fill_mod` once per modulated block
// (src/ming-dit.cc:2266-2273): a bare Linear `mods = W_ada · temb + b`
// (M = 1, N = 4H, K = adaln_dim), then folds (1 + scale) into the block's
// norm gains (nw1 = an1 · (1 + scale_msa), nw3 = fn1 · (1 + scale_mlp)).
// Every block reads the SAME temb, so all of them are one weight-streaming
// pass here: the work is reading the packed adaLN weights once (HBM-bound),
// with the few tokens riding along.
//
// Persistent warps over balanced, contiguous slices of the n_blocks * N
// weight rows (rows are contiguous in memory, so a warp's copies are whole
// coalesced rows), the next steps' copies in flight during the current
// step's math:
//
//  * Lane-per-row path (K a multiple of 256 -- the reference's 256 and the
//    [4H, 3840] shape -- and H a multiple of 32): tiles of 32 rows, each
//    lane one row, the rows streamed through a per-warp ring in shared
//    memory (one TMA per step); per 64-wide group every token's dot is an integer
//    dp4a against 8-bit limbs of its temb values (packed codes) or packed
//    fp32 FMAs (bf16 weights), temb broadcast from shared memory, no
//    cross-lane reduction (see mod_lane_kernel).
//  * Generic path (any other K): a warp per row, lanes striding over the
//    row's 16-byte chunks in fp32 FMAs, temb from shared memory, a full warp
//    reduction per row.
//
// Packed weights: a group's dequantized dot is s * sum_k q_k t_k + b * sum_k
// t_k with the codes entering as exact integers. Every token's sums are
// formed in a fixed order that does not depend on M, the grid or the row's
// position, so a row's result is the same bits whatever launch computes it
// (a CFG batch equals its per-image launches).
#include <cuda_runtime.h>

#include <atomic>

#include "mp_device.cuh"
#include "mp_kernels.h"

namespace mp {

namespace {

constexpr int kModThreads = 256;
constexpr int kModWarps = kModThreads / 32;
constexpr int kUnroll = 8;  // 16-byte loads per lane in flight per group

template <int BITS>
struct ModFmt {
  static constexpr int kPer = BITS == 0 ? 8 : (BITS == 8 ? 16 : 32);  // weights per 16-byte chunk
  static constexpr int kPairs = kPer / 2;                            // fp32 pairs per chunk
};

// Packed fp32 pair p (weights 2p, 2p + 1) of a 16-byte chunk: exact code
// values for packed codes (code_xor / magic handle signed 8-bit codes),
// the weights themselves for bf16.
template <int BITS>
__device__ __forceinline__ uint64_t chunk_pair(const uint4& c, int p, uint32_t code_xor,
                                               uint64_t neg_magic2) {
  const uint32_t words[4] = {c.x, c.y, c.z, c.w};
  if constexpr (BITS == 0) {
    const uint32_t w = words[p];
    return f32x2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  } else if constexpr (BITS == 8) {
    const uint32_t w = words[p >> 1] ^ code_xor;
    const uint32_t b0 = static_cast<uint32_t>(2 * (p & 1));
    const uint64_t q = f32x2(__uint_as_float(__byte_perm(w, 0x4Bu, 0x4550u | b0)),
                             __uint_as_float(__byte_perm(w, 0x4Bu, 0x4550u | (b0 + 1))));
    return add_f32x2(q, neg_magic2);
  } else {
    // code j of a word at bits [4j, 4j + 4): pair i of word w = codes 2i, 2i + 1,
    // the low nibble and the high nibble of byte i
    const uint32_t w = words[p >> 2];
    const uint32_t i = static_cast<uint32_t>(p & 3);
    const uint32_t ev = w & 0x0F0F0F0Fu, od = (w >> 4) & 0x0F0F0F0Fu;
    const uint64_t q = f32x2(__uint_as_float(__byte_perm(ev, 0x4Bu, 0x4550u | i)),
                             __uint_as_float(__byte_perm(od, 0x4Bu, 0x4550u | i)));
    return add_f32x2(q, neg_magic2);
  }
}

// Partial dot of one chunk with one token's temb values (pairs t2[0..kPairs)):
// two interleaved fp32 chains (even / odd weights), added at the end.
template <int BITS>
__device__ __forceinline__ float chunk_dot(const uint4& c, const uint64_t* t2, uint32_t code_xor,
                                           uint64_t neg_magic2) {
  uint64_t acc = f32x2(0.0f, 0.0f);
#pragma unroll
  for (int p = 0; p < ModFmt<BITS>::kPairs; ++p)
    acc = fma_f32x2(chunk_pair<BITS>(c, p, code_xor, neg_magic2), t2[p], acc);
  return f32x2_lo(acc) + f32x2_hi(acc);
}

// A row's bias and, for the rows whose (1 + scale) folds into a norm gain
// (chunk 0 into an1, chunk 2 into fn1), that gain (0 otherwise), as bf16 bits.
struct RowEpi {
  uint32_t bias, gain;
};

__device__ __forceinline__ RowEpi row_epi(const ModParams& p, const ModBlock& blk, int n) {
  RowEpi e;
  e.bias = __ldg(blk.bias + n);
  e.gain = 0u;
  if (n < p.H && blk.an1 != nullptr) e.gain = __ldg(blk.an1 + n);
  if (n >= 2 * p.H && n < 3 * p.H && blk.fn1 != nullptr) e.gain = __ldg(blk.fn1 + (n - 2 * p.H));
  return e;
}

// One output of a row: bias, the bf16 mods value of token m, and the
// (1 + scale) fold into the norm gain of chunks 0 and 2 of the 4H outputs.
__device__ __forceinline__ void write_token(const ModParams& p, const ModBlock& blk, int b, int n,
                                            int m, float v, RowEpi e) {
  const size_t bm = static_cast<size_t>(b) * p.m_stride + m;
  const __nv_bfloat16 mv = __float2bfloat16_rn(v + bf16_bits_to_f32(e.bias));
  reinterpret_cast<__nv_bfloat16*>(p.mods)[bm * p.N + n] = mv;
  const float scale1 = 1.0f + __bfloat162float(mv);
  if (p.nw1 != nullptr && blk.an1 != nullptr && n < p.H)
    reinterpret_cast<__nv_bfloat16*>(p.nw1)[bm * p.H + n] =
        __float2bfloat16_rn(bf16_bits_to_f32(e.gain) * scale1);
  if (p.nw3 != nullptr && blk.fn1 != nullptr && n >= 2 * p.H && n < 3 * p.H)
    reinterpret_cast<__nv_bfloat16*>(p.nw3)[bm * p.H + (n - 2 * p.H)] =
        __float2bfloat16_rn(bf16_bits_to_f32(e.gain) * scale1);
}

template <int MT>
__device__ __forceinline__ void write_row(const ModParams& p, const ModBlock& blk, int b, int n,
                                          const float* v) {
  const RowEpi e = row_epi(p, blk, n);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (m >= p.M) break;
    write_token(p, blk, b, n, m, v[m], e);
  }
}

// Balanced contiguous slice [begin, end) of `total` items for warp `w` of `nw`.
__device__ __forceinline__ void warp_slice(long long total, long long w, long long nw,
                                           long long& begin, long long& end) {
  begin = total * w / nw;
  end = total * (w + 1) / nw;
}

// ---- lane-per-row path: K a multiple of 256, H a multiple of 32 -------------
// A warp takes tiles of 32 weight rows of one block, lane r owning row r. Per
// step (the rows' next 128 bytes: 2 groups w8, 4 w4, 1 bf16) the lane reads
// its row's 16-byte chunks from the warp's ring slot and forms every token's
// dot against values all lanes read from shared memory at the same address (a
// broadcast): for packed codes integer dots (dp4a) with the token's temb
// limbs (see lane_fixed_bytes), for bf16 weights packed fp32 FMAs with its
// fp32 temb values in two interleaved chains in K order. No lane exchanges
// anything: a packed group folds in as s * sum(q t) + b * sum(t), bf16
// weights add their group sums. A token's operations do not depend on the
// launch's token count, so a row's result has the same bits in any launch (a
// CFG batch equals its per-image launches).
constexpr int kLaneRows = 32;
constexpr int kLaneTok = 8;  // tokens of one launch, at most
#ifndef MP_LANE_WARPS
#define MP_LANE_WARPS 16
#endif
constexpr int kLaneWarps = MP_LANE_WARPS;  // warps per CTA (one CTA per SM: the rings)

// A step is 128 bytes of each of the tile's 32 rows: 2 groups (w8), 4 (w4)
// or 1 (bf16).
template <int BITS>
struct LaneFmt {
  static constexpr int kGroupBytes = 64 * (BITS == 0 ? 16 : BITS) / 8;   // 128, 64, 32
  static constexpr int kRowBytes = 128;                                  // one row, one step
  static constexpr int kStepGroups = kRowBytes / kGroupBytes;
  static constexpr int kCpr = kRowBytes / 16;                            // 16-byte chunks per row
  static constexpr int kCpg = kGroupBytes / 16;                          // chunks per group
  static constexpr int kData = kLaneRows * kRowBytes;                    // one TMA box
  static constexpr int kSbRow = BITS == 0 ? 0 : 4 * kStepGroups;         // scale/bias bytes per row
  static constexpr int kSb = kLaneRows * kSbRow;
  static constexpr int kEpi = 2 * kLaneRows * 2;                         // bias, gain (bf16)
  static constexpr int kAux = (kSb + kEpi + 15) / 16 * 16;
  static constexpr int kSlot = kData + kAux + 8;                         // data, aux, barrier
  static_assert(kCpr == 8, "the 128-byte swizzle spans 8 chunks per row");
};

// A position in a warp's list of steps: rows n0 .. n0 + 31 of block b, step
// gb of the tile (advanced without divisions).
struct StepPos {
  int b, n0, gb;
  __device__ __forceinline__ void advance(int steps_per_tile, int N) {
    if (++gb == steps_per_tile) {
      gb = 0;
      n0 += kLaneRows;
      if (n0 == N) {
        n0 = 0;
        ++b;
      }
    }
  }
};

// The copies of step `pos`. lane_load_rows: lane 0 the 32 rows' 128 bytes by
// one TMA into `data` (the 128-byte swizzle puts chunk c of row r at chunk
// position c ^ (r & 7), so the lanes' row reads are conflict-free), completing
// on `bar` (needs only the block's tensor map). lane_load_aux: every lane its
// row's scale/bias words, and with the tile's last step lanes 0-7 the rows'
// bias and norm gain, into `aux` (cp.async; needs the block table).
template <int BITS>
__device__ __forceinline__ void lane_load_rows(const ModParams& p, StepPos pos, int lane,
                                               uint32_t data, uint32_t bar) {
  using L = LaneFmt<BITS>;
  if (lane == 0) {
    mbar_arrive_expect_tx(bar, L::kData);
    tma_load_2d(data, p.maps + pos.b, bar, pos.gb * (BITS == 0 ? 64 : L::kRowBytes), pos.n0);
  }
}

template <int BITS>
__device__ __forceinline__ void lane_load_aux(const ModParams& p, const ModBlock* blocks,
                                              StepPos pos, int steps_per_tile, int lane,
                                              uint32_t aux) {
  using L = LaneFmt<BITS>;
  const ModBlock& blk = blocks[pos.b];
  if constexpr (BITS != 0) {
    const uint32_t* sb =
        blk.sb + static_cast<size_t>(pos.n0 + lane) * p.sb_stride + pos.gb * L::kStepGroups;
    if constexpr (L::kSbRow == 16)
      cp_async_16(aux + lane * 16, sb);
    else
      asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(aux + lane * 8), "l"(sb)
                   : "memory");
  }
  if (pos.gb + 1 == steps_per_tile && lane < 8) {
    // lanes 0-3: bias of rows 8j .. 8j + 7; lanes 4-7: the norm gain the
    // rows' (1 + scale) folds into (chunk 0: an1, chunk 2: fn1; none otherwise)
    const uint32_t dst = aux + L::kSb + 16 * lane;
    const int part = 8 * (lane & 3);
    if (lane < 4) {
      cp_async_16(dst, blk.bias + pos.n0 + part);
    } else {
      const uint16_t* g = nullptr;
      if (pos.n0 < p.H && blk.an1 != nullptr) g = blk.an1 + pos.n0;
      if (pos.n0 >= 2 * p.H && pos.n0 < 3 * p.H && blk.fn1 != nullptr)
        g = blk.fn1 + (pos.n0 - 2 * p.H);
      if (g != nullptr) cp_async_16(dst, g + part);
    }
  }
}

__device__ __forceinline__ uint32_t pick4p(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// Packed codes take integer dot products. Each token's temb values of a
// 64-wide group (bf16: 8 significant bits) are written as integers
// T = round(t * 2^(13 - E)), E the exponent of the group's largest |t|:
// exact for every value within 6 binades of the largest, the smaller ones
// rounded to the nearest integer (an absolute error of at most 2^(E - 14),
// 2^-14 of the group's largest value; the output is rounded to bf16, 2^-9),
// and T as two signed 8-bit limbs, T = L0 + 2^8 L1 (|L1| <= 64). Then
// sum_k q_k t_k = 2^(E - 13) (A0 + 2^8 A1) with A_l = sum_k q_k L_l,k exact
// in 32-bit integers, formed four codes at a time with dp4a. Integer sums do
// not depend on their order, so a token's result is the same in any launch.
// (Three limbs, exact to 14 binades, cost a third more dp4a and limb loads:
// the w4 call is bound by its instruction stream.)
//
// Shared memory for packed codes: the block table, the limbs int8
// [MT][K / 64][kLimbs][64] (w4: within each 8 values the even ones first, as
// a code word's low nibbles hold them), per (group, token) the scale
// 2^(E - 13), the temb sum and the limb sums [K / 64][MT]; for bf16 weights
// temb as fp32 [MT][K] and nothing else. Then the warps' rings.
constexpr int kLimbs = 2;
constexpr int kLimbShift = 8 * kLimbs - 3;  // T = t * 2^(kLimbShift - E), |T| < 2^(kLimbShift + 1)
template <int BITS, int MT>
__host__ __device__ __forceinline__ size_t lane_fixed_bytes(int n_blocks, int K) {
  const size_t blk = (static_cast<size_t>(n_blocks) * sizeof(ModBlock) + 15) & ~size_t(15);
  const size_t t = BITS == 0 ? static_cast<size_t>(MT) * K * 4
                             : static_cast<size_t>(MT) * K * kLimbs +
                                   static_cast<size_t>(K / 64) * MT * (8 + 4 * kLimbs);
  return (blk + t + 127) & ~size_t(127);
}

// Position of value k (within its 64-wide group) in a limb row.
template <int BITS>
__device__ __forceinline__ int limb_pos(int k) {
  if constexpr (BITS == 4) return (k & ~7) + ((k & 1) ? 4 : 0) + ((k & 7) >> 1);
  return k;
}

// a: four unsigned 8-bit codes, b: four signed 8-bit limbs, c + sum a_i b_i.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

template <int BITS, int MT, int RING, int W>
__global__ void __launch_bounds__(32 * W, 1) mod_lane_kernel(const __grid_constant__ ModParams p) {
  using L = LaneFmt<BITS>;
  using F = ModFmt<BITS>;
  extern __shared__ __align__(128) uint8_t mod_smem[];
  ModBlock* blocks = reinterpret_cast<ModBlock*>(mod_smem);
  const size_t blk_bytes = (static_cast<size_t>(p.n_blocks) * sizeof(ModBlock) + 15) & ~size_t(15);
  const int G = p.K / 64;
  const int K4 = p.K / 4;
  float4* tq = reinterpret_cast<float4*>(mod_smem + blk_bytes);                 // bf16: [MT][K / 4]
  int8_t* tl = reinterpret_cast<int8_t*>(mod_smem + blk_bytes);                 // packed: limbs
  float* tmul = reinterpret_cast<float*>(tl + static_cast<size_t>(MT) * p.K * kLimbs);  // [G][MT]
  float* tsum = tmul + G * MT;                                                       // [G][MT]
  int* tls = reinterpret_cast<int*>(tsum + G * MT);                                  // [G][MT][kLimbs]
  const int lane = threadIdx.x & 31;
  const uint64_t neg_magic2 = f32x2(-p.code_magic, -p.code_magic);
  const int steps_per_tile = G / L::kStepGroups;
  const int tiles_per_block = p.N / kLaneRows;
  // this warp's tiles [t_begin, t_end) of the launch's n_blocks * tiles_per_block
  // (32-bit arithmetic when the products fit: 64-bit divisions cost ~1 us here)
  const long long total_tiles = static_cast<long long>(p.n_blocks) * tiles_per_block;
  const long long nwarps = static_cast<long long>(gridDim.x) * W;
  const long long gw = static_cast<long long>(blockIdx.x) * W + (threadIdx.x >> 5);
  long long t_begin, t_end;
  if (total_tiles * nwarps < (1ll << 32)) {
    const uint32_t tt = static_cast<uint32_t>(total_tiles), nw = static_cast<uint32_t>(nwarps),
                   w = static_cast<uint32_t>(gw);
    t_begin = tt * w / nw;
    t_end = tt * (w + 1u) / nw;
  } else {
    warp_slice(total_tiles, gw, nwarps, t_begin, t_end);
  }
  const bool work = t_begin < t_end;
  const int st_end = work ? static_cast<int>(t_end - t_begin) * steps_per_tile : 0;
  StepPos cpos;  // the step consumed next
  cpos.b = static_cast<int>(static_cast<uint32_t>(t_begin) / static_cast<uint32_t>(tiles_per_block));
  cpos.n0 = static_cast<int>(t_begin - static_cast<long long>(cpos.b) * tiles_per_block) * kLaneRows;
  cpos.gb = 0;
  StepPos lpos = cpos;  // the step loaded next
  // this warp's ring: RING data slots (TMA boxes, 1024-byte aligned for the
  // 128-byte swizzle), their scale/bias and epilogue words, their barriers
  const int wi = threadIdx.x >> 5;
  const uint32_t smem0 = smem_u32(mod_smem);
  const uint32_t data0 =
      (smem0 + static_cast<uint32_t>(lane_fixed_bytes<BITS, MT>(p.n_blocks, p.K)) + 1023u) & ~1023u;
  const uint32_t aux0 = data0 + static_cast<uint32_t>(W * RING * L::kData);
  const uint32_t bar0 = aux0 + static_cast<uint32_t>(W * RING * L::kAux);
  const uint32_t wdata = data0 + static_cast<uint32_t>(wi * RING * L::kData);
  const uint32_t waux = aux0 + static_cast<uint32_t>(wi * RING * L::kAux);
  const uint32_t wbar = bar0 + static_cast<uint32_t>(wi * RING * 8);
  const uint8_t* const data_p = mod_smem + (wdata - smem0);
  const uint8_t* const aux_p = mod_smem + (waux - smem0);
  if (lane == 0 && work) {
    for (int r = 0; r < RING; ++r) mbar_init(wbar + 8 * r, 1);
    fence_mbar_init();
  }
  __syncwarp();

  // global memory only once the kernels this launch depends on are done
  pdl_wait();
  pdl_release();
  // packed codes: this warp's first (group, token) temb values, loaded before
  // the copies below queue behind the first steps' weight rows
  float tp0 = 0.0f, tp1 = 0.0f;
  if constexpr (BITS != 0) {
    const int i = threadIdx.x >> 5;
    if (i < G * MT && i % MT < p.M) {
      const uint16_t* t = p.temb + static_cast<size_t>(i % MT) * p.K + (i / MT) * 64;
      tp0 = bf16_bits_to_f32(t[lane]);
      tp1 = bf16_bits_to_f32(t[32 + lane]);
    }
  }
  // prologue: the first RING - 1 steps' weight rows in flight (they need only
  // the tensor maps), then the block table, then those steps' scale/bias and
  // epilogue words (one commit group per step)
#pragma unroll 1
  for (int r = 0; r < RING - 1; ++r) {
    if (r < st_end) {
      lane_load_rows<BITS>(p, lpos, lane, wdata + r * L::kData, wbar + 8 * r);
      lpos.advance(steps_per_tile, p.N);
    }
  }
  for (int i = threadIdx.x; i < p.n_blocks; i += blockDim.x) blocks[i] = p.blocks[i];
  __syncthreads();
  {
    StepPos apos = cpos;
#pragma unroll 1
    for (int r = 0; r < RING - 1; ++r) {
      if (r < st_end) {
        lane_load_aux<BITS>(p, blocks, apos, steps_per_tile, lane, waux + r * L::kAux);
        apos.advance(steps_per_tile, p.N);
      }
      cp_async_commit();
    }
  }
  // the temb values (packed codes: their limbs) while the first steps' copies fly
  if constexpr (BITS == 0) {
    for (int i = threadIdx.x; i < MT * K4; i += blockDim.x) {
      const int m = i / K4, k4 = i - (i / K4) * K4;
      float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (m < p.M) {
        const uint16_t* t = p.temb + static_cast<size_t>(m) * p.K + 4 * k4;
        v = make_float4(bf16_bits_to_f32(t[0]), bf16_bits_to_f32(t[1]), bf16_bits_to_f32(t[2]),
                        bf16_bits_to_f32(t[3]));
      }
      tq[i] = v;
    }
  } else {
    // a warp per (group, token): lanes take values wl and 32 + wl; the
    // group's largest |t|, its limbs, the limb sums (exact integers) and the
    // temb sum (a fixed xor tree: the same bits for a token whatever else the
    // launch holds)
    const int wl = threadIdx.x & 31;
    for (int i = threadIdx.x >> 5; i < G * MT; i += W) {
      const int gi = i / MT, n = i - (i / MT) * MT;
      float t0 = tp0, t1 = tp1;  // the first pair's values are loaded
      if (i >= W && n < p.M) {
        const uint16_t* t = p.temb + static_cast<size_t>(n) * p.K + gi * 64;
        t0 = bf16_bits_to_f32(t[wl]);
        t1 = bf16_bits_to_f32(t[32 + wl]);
      } else if (i >= W) {
        t0 = t1 = 0.0f;
      }
      float amax = fmaxf(fabsf(t0), fabsf(t1));
      float v = t0 + t1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
        v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
      }
      // E: the exponent of amax (0 for an all-zero group)
      const int e = amax > 0.0f ? static_cast<int>((__float_as_uint(amax) >> 23) & 0xFFu) - 127 : 0;
      int lsum[kLimbs] = {};
      int8_t* row = tl + (static_cast<size_t>(n) * G + gi) * (64 * kLimbs);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int k = wl + 32 * h;
        int T = __float2int_rn(ldexpf(h == 0 ? t0 : t1, kLimbShift - e));
#pragma unroll
        for (int l = 0; l < kLimbs; ++l) {
          // the last limb keeps the rest (|L| <= 64); the others are the
          // signed low byte, the remainder shifted down exactly
          const int lv = l + 1 < kLimbs ? static_cast<int>(static_cast<int8_t>(T & 0xFF)) : T;
          row[64 * l + limb_pos<BITS>(k)] = static_cast<int8_t>(lv);
          lsum[l] += lv;
          T = (T - lv) >> 8;
        }
      }
#pragma unroll
      for (int l = 0; l < kLimbs; ++l)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lsum[l] += __shfl_xor_sync(0xFFFFFFFFu, lsum[l], o);
      if (wl == 0) {
        tmul[i] = ldexpf(1.0f, e - kLimbShift);
        tsum[i] = v;
#pragma unroll
        for (int l = 0; l < kLimbs; ++l) tls[kLimbs * i + l] = lsum[l];
      }
    }
  }
  __syncthreads();
  if (!work) return;
  float y[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) y[m] = 0.0f;
  int slot_c = 0, slot_l = RING - 1;  // ring slots of the consumed and the loaded step
  uint32_t dpar = 0;                  // per slot: parity of its data barrier's next phase
  for (int st = 0; st < st_end; ++st) {
    if (st + RING - 1 < st_end) {
      lane_load_rows<BITS>(p, lpos, lane, wdata + static_cast<uint32_t>(slot_l) * L::kData,
                           wbar + 8u * static_cast<uint32_t>(slot_l));
      lane_load_aux<BITS>(p, blocks, lpos, steps_per_tile, lane,
                          waux + static_cast<uint32_t>(slot_l) * L::kAux);
      lpos.advance(steps_per_tile, p.N);
    }
    slot_l = slot_l + 1 == RING ? 0 : slot_l + 1;
    cp_async_commit();
    asm volatile("cp.async.wait_group %0;" ::"n"(RING - 1) : "memory");
    {
      // the step's TMA box (bounded wait: on a timeout the error word is set
      // and the warp stops)
      const uint32_t bar = wbar + 8u * static_cast<uint32_t>(slot_c);
      const uint32_t par = (dpar >> slot_c) & 1u;
      bool ok = mbar_try_wait(bar, par);
      if (!ok) {
        const uint64_t t0 = global_timer_ns();
        while (!(ok = mbar_try_wait(bar, par)) && global_timer_ns() - t0 < p.wait_limit_ns) {
        }
      }
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        if (lane == 0) atomicOr(p.err, kErrTimeout);
        break;
      }
      dpar ^= 1u << slot_c;
    }
    __syncwarp();
    const uint8_t* slot = data_p + slot_c * L::kData;
    const uint8_t* aux = aux_p + slot_c * L::kAux;
    slot_c = slot_c + 1 == RING ? 0 : slot_c + 1;
    const uint8_t* rowp = slot + lane * L::kRowBytes;
    const int sw = lane & 7;
    uint4 sbv = make_uint4(0u, 0u, 0u, 0u);
    if constexpr (L::kSbRow == 16) {
      sbv = *reinterpret_cast<const uint4*>(aux + lane * 16);
    } else if constexpr (L::kSbRow == 8) {
      const uint2 v = *reinterpret_cast<const uint2*>(aux + lane * 8);
      sbv.x = v.x;
      sbv.y = v.y;
    }
#pragma unroll
    for (int gi = 0; gi < L::kStepGroups; ++gi) {
      const int g_abs = cpos.gb * L::kStepGroups + gi;
      if constexpr (BITS == 0) {
        // bf16 weights: packed fp32 FMAs against temb broadcast from shared memory
        const float4* tstep = tq + cpos.gb * L::kStepGroups * 16;
        uint64_t acc[MT][2];
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m][0] = acc[m][1] = f32x2(0.0f, 0.0f);
#pragma unroll
        for (int c = 0; c < L::kCpg; ++c) {
          const int ch = gi * L::kCpg + c;
          const uint4 w = *reinterpret_cast<const uint4*>(rowp + ((ch ^ sw) << 4));
          uint64_t q[F::kPairs];
#pragma unroll
          for (int pp = 0; pp < F::kPairs; ++pp) q[pp] = chunk_pair<0>(w, pp, 0u, neg_magic2);
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const float4* tm = tstep + static_cast<size_t>(m) * K4 + ch * (F::kPer / 4);
#pragma unroll
            for (int qq = 0; qq < F::kPer / 4; ++qq) {
              const float4 t = tm[qq];
              acc[m][0] = fma_f32x2(q[2 * qq], f32x2(t.x, t.y), acc[m][0]);
              acc[m][1] = fma_f32x2(q[2 * qq + 1], f32x2(t.z, t.w), acc[m][1]);
            }
          }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m)
          y[m] += (f32x2_lo(acc[m][0]) + f32x2_hi(acc[m][0])) +
                  (f32x2_lo(acc[m][1]) + f32x2_hi(acc[m][1]));
      } else {
        // packed codes: integer dots (exact in 32 bits) with the temb limbs
        // two accumulators per limb (even / odd code words) up to 4 tokens:
        // integer sums, so the split changes nothing but the dependency chains
        constexpr int kB = MT <= 4 ? MT : 1;
        int a[MT][kLimbs], b[kB][kLimbs];
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
          for (int l = 0; l < kLimbs; ++l) a[m][l] = 0;
#pragma unroll
        for (int m = 0; m < kB; ++m)
#pragma unroll
          for (int l = 0; l < kLimbs; ++l) b[m][l] = 0;
#pragma unroll
        for (int c = 0; c < L::kCpg; ++c) {
          const int ch = gi * L::kCpg + c;
          const uint4 w = *reinterpret_cast<const uint4*>(rowp + ((ch ^ sw) << 4));
          uint32_t cw[8];  // w8: 4 words of 4 codes; w4: low / high nibbles of 4 words
          if constexpr (BITS == 8) {
            cw[0] = w.x ^ p.code_xor;
            cw[1] = w.y ^ p.code_xor;
            cw[2] = w.z ^ p.code_xor;
            cw[3] = w.w ^ p.code_xor;
          } else {
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              cw[2 * i] = ws[i] & 0x0F0F0F0Fu;
              // the high nibbles in place (16 q) when they have accumulators
              // of their own (divided by 16 at the group's end, exactly):
              // one instruction fewer than shifting them down
              cw[2 * i + 1] = MT <= 4 ? ws[i] & 0xF0F0F0F0u : (ws[i] >> 4) & 0x0F0F0F0Fu;
            }
          }
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const int8_t* lr = tl + (static_cast<size_t>(m) * G + g_abs) * (64 * kLimbs) + c * F::kPer;
#pragma unroll
            for (int l = 0; l < kLimbs; ++l) {
              int& bb = MT <= 4 ? b[m < kB ? m : 0][l] : a[m][l];
              const uint4 l0 = *reinterpret_cast<const uint4*>(lr + 64 * l);
              if constexpr (BITS == 8) {
                a[m][l] = dp4a_us(cw[0], l0.x, a[m][l]);
                bb = dp4a_us(cw[1], l0.y, bb);
                a[m][l] = dp4a_us(cw[2], l0.z, a[m][l]);
                bb = dp4a_us(cw[3], l0.w, bb);
              } else {
                const uint4 l1 = *reinterpret_cast<const uint4*>(lr + 64 * l + 16);
                a[m][l] = dp4a_us(cw[0], l0.x, a[m][l]);
                bb = dp4a_us(cw[1], l0.y, bb);
                a[m][l] = dp4a_us(cw[2], l0.z, a[m][l]);
                bb = dp4a_us(cw[3], l0.w, bb);
                a[m][l] = dp4a_us(cw[4], l1.x, a[m][l]);
                bb = dp4a_us(cw[5], l1.y, bb);
                a[m][l] = dp4a_us(cw[6], l1.z, a[m][l]);
                bb = dp4a_us(cw[7], l1.w, bb);
              }
            }
          }
        }
        const uint32_t sbw = pick4p(sbv, gi);
        const float sc = bf16_bits_to_f32(sbw & 0xFFFFu), bi = bf16_bits_to_f32(sbw >> 16);
        const int off = p.code_xor != 0u ? 128 : 0;  // signed codes entered as q + 128
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const int i = g_abs * MT + m;
          int sl[kLimbs];
#pragma unroll
          for (int l = 0; l < kLimbs; ++l)
            sl[l] = (MT <= 4 ? a[m][l] + (BITS == 4 ? b[m < kB ? m : 0][l] >> 4 : b[m < kB ? m : 0][l])
                             : a[m][l]) -
                    off * tls[kLimbs * i + l];
          float dsum = static_cast<float>(sl[kLimbs - 1]);
#pragma unroll
          for (int l = kLimbs - 2; l >= 0; --l) dsum = __fmaf_rn(256.0f, dsum, static_cast<float>(sl[l]));
          const float d = __fmul_rn(dsum, tmul[i]);
          y[m] += __fmaf_rn(sc, d, __fmul_rn(bi, tsum[i]));
        }
      }
    }
    if (cpos.gb + 1 == steps_per_tile) {
      // the tile's rows are complete: row n0 + lane for every token
      const int b = cpos.b, n = cpos.n0 + lane;
      const uint16_t* epi = reinterpret_cast<const uint16_t*>(aux + L::kSb);
      const bool has_gain = (cpos.n0 < p.H && blocks[b].an1 != nullptr) ||
                            (cpos.n0 >= 2 * p.H && cpos.n0 < 3 * p.H && blocks[b].fn1 != nullptr);
      RowEpi e;
      e.bias = epi[lane];
      e.gain = has_gain ? epi[kLaneRows + lane] : 0u;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m < p.M) write_token(p, blocks[b], b, n, m, y[m], e);
        y[m] = 0.0f;
      }
    }
    cpos.advance(steps_per_tile, p.N);
    __syncwarp();  // every lane has read the slot before a later step's copies reuse it
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// ---- generic path: a warp per row -------------------------------------------
// Shared memory: the block table, then temb as fp32 in a chunk-interleaved
// layout ([token][quad of the chunk][chunk][4]: lanes reading consecutive
// chunks read consecutive 16-byte words), then the per-chunk temb sums.
template <int BITS, int MT>
__global__ void __launch_bounds__(kModThreads) mod_warp_kernel(const __grid_constant__ ModParams p) {
  using F = ModFmt<BITS>;
  constexpr int Q = F::kPer / 4;  // float quads per chunk
  extern __shared__ uint8_t mod_smem[];
  pdl_wait();
  pdl_release();
  ModBlock* blocks = reinterpret_cast<ModBlock*>(mod_smem);
  const int row_bytes = BITS == 0 ? p.K * 2 : p.K * BITS / 8;
  const int C = row_bytes / 16;
  const size_t blk_bytes = (static_cast<size_t>(p.n_blocks) * sizeof(ModBlock) + 15) & ~size_t(15);
  float4* tq = reinterpret_cast<float4*>(mod_smem + blk_bytes);
  float* tsum = reinterpret_cast<float*>(tq + static_cast<size_t>(MT) * Q * C);
  for (int i = threadIdx.x; i < p.n_blocks; i += blockDim.x) blocks[i] = p.blocks[i];
  for (int i = threadIdx.x; i < MT * Q * C; i += blockDim.x) {
    const int m = i / (Q * C), rem = i % (Q * C), q = rem / C, ch = rem % C;
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (m < p.M) {
      const uint16_t* t = p.temb + static_cast<size_t>(m) * p.K + ch * F::kPer + 4 * q;
      v = make_float4(bf16_bits_to_f32(t[0]), bf16_bits_to_f32(t[1]), bf16_bits_to_f32(t[2]),
                      bf16_bits_to_f32(t[3]));
    }
    tq[i] = v;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < MT * C; i += blockDim.x) {
    const int m = i / C, ch = i % C;
    float s = 0.0f;
    for (int q = 0; q < Q; ++q) {
      const float4 v = tq[(m * Q + q) * C + ch];
      s += v.x;
      s += v.y;
      s += v.z;
      s += v.w;
    }
    tsum[i] = s;
  }
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const uint64_t neg_magic2 = f32x2(-p.code_magic, -p.code_magic);
  const long long total_rows = static_cast<long long>(p.n_blocks) * p.N;
  const long long nwarps = static_cast<long long>(gridDim.x) * kModWarps;
  const long long gw = static_cast<long long>(blockIdx.x) * kModWarps + (threadIdx.x >> 5);
  long long r_begin, r_end;
  warp_slice(total_rows, gw, nwarps, r_begin, r_end);
  int b = static_cast<int>(r_begin / p.N);
  int n = static_cast<int>(r_begin - static_cast<long long>(b) * p.N);
  for (long long r = r_begin; r < r_end; ++r, n = (n + 1 == p.N ? 0 : n + 1), b += (n == 0)) {
    const ModBlock& blk = blocks[b];
    const uint8_t* row = blk.w + static_cast<size_t>(n) * row_bytes;
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
    for (int ch0 = 0; ch0 < C; ch0 += 32 * kUnroll) {
      uint4 c[kUnroll];
      uint32_t sbw[kUnroll];
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) {
        const int ch = ch0 + 32 * j + lane;
        c[j] = make_uint4(0u, 0u, 0u, 0u);
        sbw[j] = 0u;
        if (ch < C) {
          c[j] = ld_global_nc_v4(row + static_cast<size_t>(ch) * 16);
          if (BITS != 0)
            sbw[j] = __ldg(blk.sb + static_cast<size_t>(n) * p.sb_stride + (ch * F::kPer) / 64);
        }
      }
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) {
        const int ch = ch0 + 32 * j + lane;
        if (ch >= C) continue;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          uint64_t t2[F::kPairs];
#pragma unroll
          for (int q = 0; q < Q; ++q) {
            const float4 v = tq[(m * Q + q) * C + ch];
            t2[2 * q] = f32x2(v.x, v.y);
            t2[2 * q + 1] = f32x2(v.z, v.w);
          }
          const float d = chunk_dot<BITS>(c[j], t2, p.code_xor, neg_magic2);
          if constexpr (BITS == 0) {
            acc[m] += d;
          } else {
            const float sc = bf16_bits_to_f32(sbw[j] & 0xFFFFu);
            const float bi = bf16_bits_to_f32(sbw[j] >> 16);
            acc[m] += fmaf(sc, d, bi * tsum[m * C + ch]);
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xFFFFFFFFu, acc[m], o);
    if (lane == 0) write_row<MT>(p, blk, b, n, acc);
  }
}

// Resident CTAs per SM of a kernel at `smem` bytes (looked up once per device).
template <typename K>
int resident_ctas(K kernel, int threads, size_t smem, std::atomic<int>* cache) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  int per_sm = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) !=
          cudaSuccess ||
      per_sm <= 0) {
    (void)cudaGetLastError();
    per_sm = 1;
  }
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    sms = 1;
  v = per_sm * sms;
  cache[dev].store(v, std::memory_order_relaxed);
  return v;
}

template <typename K>
cudaError_t launch_persistent(K kernel, int threads, const ModParams& p, size_t smem,
                              long long work_warps, std::atomic<int>* cache, cudaStream_t stream) {
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const int warps = threads / 32;
  const long long want = (work_warps + warps - 1) / warps;
  const long long most = resident_ctas(kernel, threads, smem, cache);
  const int grid = static_cast<int>(want < most ? (want > 0 ? want : 1) : most);
  // may begin while the previous kernel on the stream finishes (the kernel
  // waits for it before touching global memory)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int BITS, int MT>
cudaError_t launch_mod_warp(const ModParams& p, cudaStream_t stream) {
  const int row_bytes = BITS == 0 ? p.K * 2 : p.K * BITS / 8;
  const int C = row_bytes / 16;
  const size_t blk_bytes = (static_cast<size_t>(p.n_blocks) * sizeof(ModBlock) + 15) & ~size_t(15);
  const long long rows = static_cast<long long>(p.n_blocks) * p.N;
  constexpr int Q = ModFmt<BITS>::kPer / 4;
  const size_t smem = blk_bytes + static_cast<size_t>(MT) * Q * C * 16 + static_cast<size_t>(MT) * C * 4;
  static std::atomic<int> cache[64];
  return launch_persistent(mod_warp_kernel<BITS, MT>, kModThreads, p, smem, rows, cache, stream);
}

constexpr size_t kModSmemLimit = 227 * 1024;

template <int BITS, int MT, int RING, int W>
cudaError_t launch_mod_lane_ring(const ModParams& p, cudaStream_t stream) {
  const size_t smem = lane_fixed_bytes<BITS, MT>(p.n_blocks, p.K) + 1024 +
                      static_cast<size_t>(W) * RING * LaneFmt<BITS>::kSlot;
  const long long tiles = static_cast<long long>(p.n_blocks) * p.N / kLaneRows;
  static std::atomic<int> cache[64];
  return launch_persistent(mod_lane_kernel<BITS, MT, RING, W>, 32 * W, p, smem, tiles, cache,
                           stream);
}

// Packed codes for one or two tokens take kLaneWarpsWide warps per CTA with
// two-slot rings when those fit (the w4 call is paced by its instruction
// stream, and more warps hide its shared-memory and dp4a latencies: K 256,
// w4 M = 1 22.5 -> 20.7 us, M = 2 28.7 -> 26.7 us, w8 M = 1 30.8 -> 28.7 us);
// more tokens per launch need the registers of kLaneWarps warps. Otherwise
// the deepest ring (steps in flight per warp, 6 at most) that fits the
// shared memory beside the block table and the temb copy (which grows with K).
constexpr int kLaneWarpsWide = 24;
template <int BITS, int MT>
cudaError_t launch_mod_lane(const ModParams& p, cudaStream_t stream) {
  const size_t fixed = lane_fixed_bytes<BITS, MT>(p.n_blocks, p.K);
  auto fits = [&](int warps, int ring) {
    return fixed + 1024 + static_cast<size_t>(warps) * ring * LaneFmt<BITS>::kSlot <=
           kModSmemLimit;
  };
  if constexpr (BITS != 0 && MT <= 2) {
    if (fits(kLaneWarpsWide, 2)) return launch_mod_lane_ring<BITS, MT, 2, kLaneWarpsWide>(p, stream);
  }
  if (fits(kLaneWarps, 6)) return launch_mod_lane_ring<BITS, MT, 6, kLaneWarps>(p, stream);
  if (fits(kLaneWarps, 4)) return launch_mod_lane_ring<BITS, MT, 4, kLaneWarps>(p, stream);
  if (fits(kLaneWarps, 3)) return launch_mod_lane_ring<BITS, MT, 3, kLaneWarps>(p, stream);
  if (fits(kLaneWarps, 2)) return launch_mod_lane_ring<BITS, MT, 2, kLaneWarps>(p, stream);
  return cudaErrorInvalidValue;
}

// K a multiple of 256 and H of 32 (the 32 rows of a tile share a block and a
// chunk of the 4H outputs).
bool lane_shape(int n, int k) { return k % 256 == 0 && n % (4 * kLaneRows) == 0; }

// Token counts round up to 1, 2, 4 or 8 (registers scale with it; a token's
// bits do not).
template <int BITS>
cudaError_t launch_mod_bits(const ModParams& p, cudaStream_t stream) {
  if (lane_shape(p.N, p.K)) {
    if (p.maps == nullptr || p.err == nullptr) return cudaErrorInvalidValue;
    if (p.M > kLaneTok) return cudaErrorInvalidValue;
    if (p.M == 1) return launch_mod_lane<BITS, 1>(p, stream);
    if (p.M == 2) return launch_mod_lane<BITS, 2>(p, stream);
    if (p.M <= 4) return launch_mod_lane<BITS, 4>(p, stream);
    return launch_mod_lane<BITS, 8>(p, stream);
  }
  if (p.M > kModMaxTok) return cudaErrorInvalidValue;
  if (p.M == 1) return launch_mod_warp<BITS, 1>(p, stream);
  if (p.M == 2) return launch_mod_warp<BITS, 2>(p, stream);
  return launch_mod_warp<BITS, 4>(p, stream);
}

}  // namespace

// Tokens of one launch: on the lane path as many (up to 8) as leave room for
// a two-slot ring beside the fp32 temb copy.
int mod_tokens_per_launch(int n, int k, int n_blocks) {
  if (!lane_shape(n, k)) return kModMaxTok;
  size_t slot = LaneFmt<8>::kSlot;
  if (LaneFmt<4>::kSlot > slot) slot = LaneFmt<4>::kSlot;
  if (LaneFmt<0>::kSlot > slot) slot = LaneFmt<0>::kSlot;
  const size_t ring2 = 1024 + static_cast<size_t>(kLaneWarps) * 2 * slot;  // with the alignment
  for (int mt = kLaneTok; mt > 1; mt >>= 1) {
    const size_t blk = (static_cast<size_t>(n_blocks) * sizeof(ModBlock) + 15) & ~size_t(15);
    const size_t fixed = (blk + static_cast<size_t>(mt) * k * 4 + static_cast<size_t>(k / 64) * mt * 4 +
                          127) & ~size_t(127);
    if (fixed + ring2 <= kModSmemLimit) return mt;
  }
  return 1;
}

cudaError_t launch_mod(const ModParams& p, cudaStream_t stream) {
  const int row_bytes = p.bits == 0 ? p.K * 2 : p.K * p.bits / 8;
  if (row_bytes % 16 != 0 || p.M < 1 || p.m_stride < p.M) return cudaErrorInvalidValue;
  if (p.bits != 0 && p.K % 64 != 0) return cudaErrorInvalidValue;
  if (p.bits == 8) return launch_mod_bits<8>(p, stream);
  if (p.bits == 4) return launch_mod_bits<4>(p, stream);
  return launch_mod_bits<0>(p, stream);
}

}  // namespace mp
