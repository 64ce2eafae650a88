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
// weight rows (rows are contiguous in memory, so a warp reads whole rows with
// coalesced loads), the next step's loads issued before the current step's
// math:
//
//  * Tensor-core path (K a multiple of 256 -- the reference's 256 and the
//    [4H, 3840] shape -- and N a multiple of 64): tiles of 16 rows; per
//    64-wide group the dot products with up to 8 tokens are mma.sync
//    m16n8k16 with the weights as the A fragment (packed codes become exact
//    fp16 integers) and the tokens' temb as the B fragment (see
//    mod_mma_kernel).
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

#include <cuda_fp16.h>

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

// ---- tensor-core path: K a multiple of 256, N a multiple of 64 --------------
// A warp takes tiles of 16 weight rows; per 64-wide K group each lane reads
// the 16 consecutive weights [16q, 16q + 16) of the group (q = lane % 4) of
// rows g and g + 8 (g = lane / 4): w8 16 bytes, w4 8 bytes, bf16 32 bytes.
// The group's dot products with up to 8 tokens are four mma.sync m16n8k16:
// the lane's weights are the A fragment (packed codes become exact fp16
// integers: one byte-permute makes two 1024 + q halves, one half subtraction
// removes the 1024; bf16 weights are used as they are), the tokens' temb
// values the B fragment (the same permutation of K, built once per CTA in
// shared memory; fp16 for packed weights, so temb must lie within fp16's
// range, |t| < 65504), fp32 accumulation. A packed group is summed on its own
// and folded in as s * sum(q t) + b * sum(t) (the temb sums per group and
// token also in shared memory); bf16 weights accumulate over all of K. Each
// token is one MMA column, computed the same way whatever the other columns
// hold.
constexpr int kMmaTok = 8;     // tokens of one launch (the MMA's N)
constexpr int kGroupsPerStep = 4;

template <int BITS>
struct MmaFmt {
  // bytes of one lane's slice of one row's group
  static constexpr int kLaneBytes = BITS == 0 ? 32 : (BITS == 8 ? 16 : 8);
  static constexpr int kWords = kLaneBytes / 4;
  static constexpr int kGroupBytes = 4 * kLaneBytes;
};

// K offsets (within a group) of the A slots (a0 low, a0 high, a2 low, a2
// high) of k-step s for quad q: the lane's weights in the order its packed
// words give them.
template <int BITS>
__device__ __forceinline__ void mma_kslots(int s, int q, int (&k)[4]) {
  if constexpr (BITS == 4) {
    const int base = 16 * q + 8 * (s >> 1) + 4 * (s & 1);
    k[0] = base; k[1] = base + 2; k[2] = base + 1; k[3] = base + 3;
  } else {
    const int base = 16 * q + 4 * s;
    k[0] = base; k[1] = base + 1; k[2] = base + 2; k[3] = base + 3;
  }
}

__device__ __forceinline__ uint32_t half2_bits_of(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// A-fragment words (the a0 / a2 halves) of k-step s from a lane's words w[]:
// two weights each, as f16x2 exact integers (packed) or bf16x2 (dense).
template <int BITS>
__device__ __forceinline__ void mma_afrag(const uint32_t* w, int s, uint32_t code_xor,
                                          uint32_t magic2, uint32_t& lo, uint32_t& hi) {
  if constexpr (BITS == 0) {
    lo = w[2 * s];
    hi = w[2 * s + 1];
  } else {
    uint32_t x0, x1;
    if constexpr (BITS == 8) {
      const uint32_t v = w[s] ^ code_xor;
      x0 = __byte_perm(v, 0x64u, 0x4140u);  // codes 0, 1 of the word
      x1 = __byte_perm(v, 0x64u, 0x4342u);  // codes 2, 3
    } else {
      const uint32_t v = w[s >> 1];
      const uint32_t ev = v & 0x0F0F0F0Fu, od = (v >> 4) & 0x0F0F0F0Fu;
      const uint32_t sel = (s & 1) ? 0x4342u : 0x4140u;
      x0 = __byte_perm(ev, 0x64u, sel);  // codes 4h, 4h + 2 (h = s & 1)
      x1 = __byte_perm(od, 0x64u, sel);  // codes 4h + 1, 4h + 3
    }
    __half2 h0 = __hsub2(*reinterpret_cast<__half2*>(&x0), *reinterpret_cast<const __half2*>(&magic2));
    __half2 h1 = __hsub2(*reinterpret_cast<__half2*>(&x1), *reinterpret_cast<const __half2*>(&magic2));
    lo = *reinterpret_cast<uint32_t*>(&h0);
    hi = *reinterpret_cast<uint32_t*>(&h1);
  }
}

template <int BITS>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (BITS == 0) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// Each warp streams its steps (16 rows x kGroupsPerStep groups) through a
// private ring of RING slots in shared memory with 16-byte cp.async copies,
// RING - 1 steps in flight: a slot holds the step's weights (16 rows, the
// 16-byte chunks of a row XOR-swizzled so the lanes' fragment reads are
// conflict-free), the rows' scale/bias words of the step's groups, and with
// the tile's last step the rows' bias and norm gain.
template <int BITS>
struct RingFmt {
  static constexpr int kRowBytes = kGroupsPerStep * MmaFmt<BITS>::kGroupBytes;  // one row, one step
  static constexpr int kCpr = kRowBytes / 16;                                   // 16-byte chunks per row
  static constexpr int kData = 16 * kRowBytes;
  static constexpr int kSb = BITS == 0 ? 0 : 16 * 16;
  static constexpr int kSlot = ((kData + kSb + 64) + 127) / 128 * 128;
  __device__ static __forceinline__ int swz(int row) {
    return BITS == 8 ? 4 * (row & 1) : (BITS == 4 ? 2 * (row & 3) : (row & 1));
  }
};

// A position in a warp's list of steps: tile rows n0 .. n0 + 15 of block b,
// step gb of the tile (advanced without divisions).
struct StepPos {
  int b, n0, gb;
  __device__ __forceinline__ void advance(int steps_per_tile, int N) {
    if (++gb == steps_per_tile) {
      gb = 0;
      n0 += 16;
      if (n0 == N) {
        n0 = 0;
        ++b;
      }
    }
  }
};

// Issues the copies of step `pos` into `slot` (this lane's share).
template <int BITS>
__device__ __forceinline__ void ring_load(const ModParams& p, const ModBlock* blocks, StepPos pos,
                                          int lane, uint32_t slot) {
  using R = RingFmt<BITS>;
  const int b = pos.b, n0 = pos.n0, gb = pos.gb;
  const ModBlock& blk = blocks[b];
  const size_t row_bytes = static_cast<size_t>(p.K) * (BITS == 0 ? 16 : BITS) / 8;
  const uint8_t* src = blk.w + static_cast<size_t>(n0) * row_bytes + static_cast<size_t>(gb) * R::kRowBytes;
#pragma unroll
  for (int c = lane; c < 16 * R::kCpr; c += 32) {
    const int row = c / R::kCpr, cc = c % R::kCpr;
    cp_async_16(slot + row * R::kRowBytes + ((cc ^ R::swz(row)) << 4),
                src + static_cast<size_t>(row) * row_bytes + cc * 16);
  }
  if constexpr (BITS != 0) {
    if (lane < 16)
      cp_async_16(slot + R::kData + lane * 16,
                  blk.sb + static_cast<size_t>(n0 + lane) * p.sb_stride + gb * kGroupsPerStep);
  }
  if ((gb + 1) * kGroupsPerStep * 64 == p.K && lane >= 16 && lane < 20) {
    // the tile's last step: bias of its 16 rows, and the norm gain their
    // (1 + scale) folds into (chunk 0: an1, chunk 2: fn1; none otherwise)
    const uint32_t dst = slot + R::kData + R::kSb + 16 * (lane - 16);
    const int half = (lane & 1) * 8;
    if (lane < 18) {
      cp_async_16(dst, blk.bias + n0 + half);
    } else {
      const uint16_t* g = nullptr;
      if (n0 < p.H && blk.an1 != nullptr) g = blk.an1 + n0;
      if (n0 >= 2 * p.H && n0 < 3 * p.H && blk.fn1 != nullptr) g = blk.fn1 + (n0 - 2 * p.H);
      if (g != nullptr) cp_async_16(dst, g + half);
    }
  }
}

// The lane's weights of (row, group gi) from a slot (a pointer into shared
// memory), as the words mma_afrag takes.
template <int BITS>
__device__ __forceinline__ void ring_words(const uint8_t* slot, int row, int gi, int q,
                                           uint32_t (&w)[MmaFmt<BITS>::kWords]) {
  using R = RingFmt<BITS>;
  const uint8_t* rb = slot + row * R::kRowBytes;
  if constexpr (BITS == 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(rb + (((gi * 4 + q) ^ R::swz(row)) << 4));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (BITS == 4) {
    const uint2 v = *reinterpret_cast<const uint2*>(
        rb + (((gi * 2 + (q >> 1)) ^ R::swz(row)) << 4) + (q & 1) * 8);
    w[0] = v.x; w[1] = v.y;
  } else {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(rb + (((gi * 8 + 2 * q + c) ^ R::swz(row)) << 4));
      w[4 * c] = v.x; w[4 * c + 1] = v.y; w[4 * c + 2] = v.z; w[4 * c + 3] = v.w;
    }
  }
}

__device__ __forceinline__ uint32_t pick4p(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

template <int BITS, int RING>
__global__ void __launch_bounds__(kModThreads) mod_mma_kernel(const __grid_constant__ ModParams p) {
  using R = RingFmt<BITS>;
  extern __shared__ __align__(128) uint8_t mod_smem[];
  ModBlock* blocks = reinterpret_cast<ModBlock*>(mod_smem);
  const size_t blk_bytes = (static_cast<size_t>(p.n_blocks) * sizeof(ModBlock) + 15) & ~size_t(15);
  const int G = p.K / 64;
  uint2* bfrag = reinterpret_cast<uint2*>(mod_smem + blk_bytes);       // [G][4][32]
  float* tsum = reinterpret_cast<float*>(bfrag + static_cast<size_t>(G) * 4 * 32);  // [G][8]
  const size_t ring_off = (blk_bytes + static_cast<size_t>(G) * 4 * 32 * 8 +
                           static_cast<size_t>(G) * kMmaTok * 4 + 127) & ~size_t(127);
  for (int i = threadIdx.x; i < p.n_blocks; i += blockDim.x) blocks[i] = p.blocks[i];
  for (int i = threadIdx.x; i < G * 4 * 32; i += blockDim.x) {
    const int gi = i >> 7, s = (i >> 5) & 3, ln = i & 31;
    const int n = ln >> 2, q = ln & 3;
    int k[4];
    mma_kslots<BITS>(s, q, k);
    uint16_t tb[4] = {0, 0, 0, 0};
    if (n < p.M)
      for (int j = 0; j < 4; ++j) tb[j] = p.temb[static_cast<size_t>(n) * p.K + gi * 64 + k[j]];
    uint2 v;
    if constexpr (BITS == 0) {
      v.x = static_cast<uint32_t>(tb[0]) | (static_cast<uint32_t>(tb[1]) << 16);
      v.y = static_cast<uint32_t>(tb[2]) | (static_cast<uint32_t>(tb[3]) << 16);
    } else {
      v.x = half2_bits_of(bf16_bits_to_f32(tb[0]), bf16_bits_to_f32(tb[1]));
      v.y = half2_bits_of(bf16_bits_to_f32(tb[2]), bf16_bits_to_f32(tb[3]));
    }
    bfrag[i] = v;
  }
  if constexpr (BITS != 0) {
    // per (group, token) the sum of its 64 temb values: a warp each, lanes
    // adding two values, then a fixed xor tree (the same bits for a token
    // whatever else the launch holds)
    const int wl = threadIdx.x & 31;
    for (int i = threadIdx.x >> 5; i < G * kMmaTok; i += kModWarps) {
      const int gi = i / kMmaTok, n = i % kMmaTok;
      float v = 0.0f;
      if (n < p.M) {
        const uint16_t* t = p.temb + static_cast<size_t>(n) * p.K + gi * 64;
        v = bf16_bits_to_f32(t[wl]) + bf16_bits_to_f32(t[32 + wl]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
      if (wl == 0) tsum[i] = v;
    }
  }
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int q = lane & 3, g = lane >> 2;
  const uint32_t code_xor = p.code_xor;
  // 1024 (affine) or 1152 (signed 8-bit codes, offset by 128), as f16x2
  const uint32_t magic2 = code_xor != 0u ? 0x64806480u : 0x64006400u;
  const int steps_per_tile = G / kGroupsPerStep;
  const long long total_tiles = static_cast<long long>(p.n_blocks) * p.N / 16;
  const long long nwarps = static_cast<long long>(gridDim.x) * kModWarps;
  const long long gw = static_cast<long long>(blockIdx.x) * kModWarps + (threadIdx.x >> 5);
  long long t_begin, t_end;
  warp_slice(total_tiles, gw, nwarps, t_begin, t_end);
  if (t_begin >= t_end) return;
  const int st_end = static_cast<int>(t_end - t_begin) * steps_per_tile;
  const int tiles_per_block = p.N / 16;
  StepPos cpos;  // the step consumed next
  cpos.b = static_cast<int>(t_begin / tiles_per_block);
  cpos.n0 = static_cast<int>(t_begin - static_cast<long long>(cpos.b) * tiles_per_block) * 16;
  cpos.gb = 0;
  StepPos lpos = cpos;  // the step loaded next
  uint8_t* const ring_p = mod_smem + ring_off + (threadIdx.x >> 5) * RING * R::kSlot;
  const uint32_t ring = smem_u32(ring_p);

  // prologue: the first RING - 1 steps in flight (one commit group per step)
#pragma unroll 1
  for (int r = 0; r < RING - 1; ++r) {
    if (r < st_end) {
      ring_load<BITS>(p, blocks, lpos, lane, ring + r * R::kSlot);
      lpos.advance(steps_per_tile, p.N);
    }
    cp_async_commit();
  }
  float y[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // rows g, g + 8 x tokens 2q, 2q + 1
  int slot_c = 0, slot_l = RING - 1;  // ring slots of the consumed and the loaded step
  for (int st = 0; st < st_end; ++st) {
    if (st + RING - 1 < st_end) {
      ring_load<BITS>(p, blocks, lpos, lane, ring + static_cast<uint32_t>(slot_l) * R::kSlot);
      lpos.advance(steps_per_tile, p.N);
    }
    slot_l = slot_l + 1 == RING ? 0 : slot_l + 1;
    cp_async_commit();
    asm volatile("cp.async.wait_group %0;" ::"n"(RING - 1) : "memory");
    __syncwarp();
    const uint8_t* slot = ring_p + slot_c * R::kSlot;
    slot_c = slot_c + 1 == RING ? 0 : slot_c + 1;
    const int gb = cpos.gb;
    uint4 sb0 = make_uint4(0u, 0u, 0u, 0u), sb1 = sb0;
    if constexpr (BITS != 0) {
      sb0 = *reinterpret_cast<const uint4*>(slot + R::kData + g * 16);
      sb1 = *reinterpret_cast<const uint4*>(slot + R::kData + (g + 8) * 16);
    }
#pragma unroll
    for (int gi = 0; gi < kGroupsPerStep; ++gi) {
      const int g_abs = gb * kGroupsPerStep + gi;
      uint32_t w0[MmaFmt<BITS>::kWords], w1[MmaFmt<BITS>::kWords];
      ring_words<BITS>(slot, g, gi, q, w0);
      ring_words<BITS>(slot, g + 8, gi, q, w1);
      float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // the group's own sums (independent chains)
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        uint32_t a0, a2, a1, a3;
        mma_afrag<BITS>(w0, s, code_xor, magic2, a0, a2);
        mma_afrag<BITS>(w1, s, code_xor, magic2, a1, a3);
        const uint2 b = bfrag[(g_abs * 4 + s) * 32 + lane];
        mma_16816<BITS>(c, a0, a1, a2, a3, b.x, b.y);
      }
      if constexpr (BITS == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) y[j] += c[j];
      } else {
        const uint32_t sw0 = pick4p(sb0, gi), sw1 = pick4p(sb1, gi);
        const float2 ts = *reinterpret_cast<const float2*>(&tsum[g_abs * kMmaTok + 2 * q]);
        const float s0 = bf16_bits_to_f32(sw0 & 0xFFFFu), b0 = bf16_bits_to_f32(sw0 >> 16);
        const float s1 = bf16_bits_to_f32(sw1 & 0xFFFFu), b1 = bf16_bits_to_f32(sw1 >> 16);
        y[0] += fmaf(s0, c[0], b0 * ts.x);
        y[1] += fmaf(s0, c[1], b0 * ts.y);
        y[2] += fmaf(s1, c[2], b1 * ts.x);
        y[3] += fmaf(s1, c[3], b1 * ts.y);
      }
    }
    if (gb + 1 == steps_per_tile) {
      // the tile's rows are complete: rows g and g + 8, tokens 2q and 2q + 1
      const int b = cpos.b, n0 = cpos.n0;
      const bool has_gain = (n0 < p.H && blocks[b].an1 != nullptr) ||
                            (n0 >= 2 * p.H && n0 < 3 * p.H && blocks[b].fn1 != nullptr);
      for (int h = 0; h < 2; ++h) {
        const int rr = g + 8 * h;
        const uint16_t* epi = reinterpret_cast<const uint16_t*>(slot + R::kData + R::kSb);
        RowEpi e;
        e.bias = epi[rr];
        e.gain = has_gain ? epi[16 + rr] : 0u;
        for (int ee = 0; ee < 2; ++ee) {
          const int m = 2 * q + ee;
          if (m < p.M) write_token(p, blocks[b], b, n0 + rr, m, y[2 * h + ee], e);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) y[j] = 0.0f;
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
int resident_ctas(K kernel, size_t smem, std::atomic<int>* cache) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  int per_sm = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kModThreads, smem) !=
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
cudaError_t launch_persistent(K kernel, const ModParams& p, size_t smem, long long work_warps,
                              std::atomic<int>* cache, cudaStream_t stream) {
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const long long want = (work_warps + kModWarps - 1) / kModWarps;
  const long long most = resident_ctas(kernel, smem, cache);
  const int grid = static_cast<int>(want < most ? (want > 0 ? want : 1) : most);
  kernel<<<grid, kModThreads, smem, stream>>>(p);
  return cudaGetLastError();
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
  return launch_persistent(mod_warp_kernel<BITS, MT>, p, smem, rows, cache, stream);
}

template <int BITS, int RING>
cudaError_t launch_mod_mma_ring(const ModParams& p, size_t fixed, cudaStream_t stream) {
  const size_t smem = fixed + static_cast<size_t>(kModWarps) * RING * RingFmt<BITS>::kSlot;
  const long long tiles = static_cast<long long>(p.n_blocks) * p.N / 16;
  static std::atomic<int> cache[64];
  return launch_persistent(mod_mma_kernel<BITS, RING>, p, smem, tiles, cache, stream);
}

// The deepest ring (steps in flight per warp) that fits the shared memory
// beside the block table and the B fragments (which grow with K).
template <int BITS>
cudaError_t launch_mod_mma(const ModParams& p, cudaStream_t stream) {
  constexpr int kDeep = BITS == 4 ? 9 : (BITS == 8 ? 5 : 3);
  const size_t blk_bytes = (static_cast<size_t>(p.n_blocks) * sizeof(ModBlock) + 15) & ~size_t(15);
  const int G = p.K / 64;
  const size_t fixed = (blk_bytes + static_cast<size_t>(G) * 4 * 32 * 8 +
                        static_cast<size_t>(G) * kMmaTok * 4 + 127) & ~size_t(127);
  constexpr size_t kLimit = 227 * 1024;
  auto fits = [&](int ring, int slot) {
    return fixed + static_cast<size_t>(kModWarps) * ring * slot <= kLimit;
  };
  if (fits(kDeep, RingFmt<BITS>::kSlot)) return launch_mod_mma_ring<BITS, kDeep>(p, fixed, stream);
  if (fits(3, RingFmt<BITS>::kSlot)) return launch_mod_mma_ring<BITS, 3>(p, fixed, stream);
  if (fits(2, RingFmt<BITS>::kSlot)) return launch_mod_mma_ring<BITS, 2>(p, fixed, stream);
  return cudaErrorInvalidValue;
}

// K a multiple of 256 and N of 64 (so the 16 rows of a tile share a block and
// a chunk of the 4H outputs)
bool mma_shape(int n, int k) { return k % (64 * kGroupsPerStep) == 0 && n % 64 == 0; }

// The generic path's token count rounded up to 1, 2 or 4: registers scale with it.
template <int BITS>
cudaError_t launch_mod_bits(const ModParams& p, cudaStream_t stream) {
  if (mma_shape(p.N, p.K)) {
    if (p.M > kMmaTok) return cudaErrorInvalidValue;
    return launch_mod_mma<BITS>(p, stream);
  }
  if (p.M > kModMaxTok) return cudaErrorInvalidValue;
  if (p.M == 1) return launch_mod_warp<BITS, 1>(p, stream);
  if (p.M == 2) return launch_mod_warp<BITS, 2>(p, stream);
  return launch_mod_warp<BITS, 4>(p, stream);
}

}  // namespace

int mod_tokens_per_launch(int n, int k) { return mma_shape(n, k) ? kMmaTok : kModMaxTok; }

cudaError_t launch_mod(const ModParams& p, cudaStream_t stream) {
  const int row_bytes = p.bits == 0 ? p.K * 2 : p.K * p.bits / 8;
  if (row_bytes % 16 != 0 || p.M < 1 || p.m_stride < p.M) return cudaErrorInvalidValue;
  if (p.bits != 0 && p.K % 64 != 0) return cudaErrorInvalidValue;
  if (p.bits == 8) return launch_mod_bits<8>(p, stream);
  if (p.bits == 4) return launch_mod_bits<4>(p, stream);
  return launch_mod_bits<0>(p, stream);
}

}  // namespace mp
