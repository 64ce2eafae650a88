// Batched adaLN modulation for all modulated blocks in ONE launch.
//
// The reference runs `fill_mod` once per modulated block
// (src/ming-dit.cc:2266-2273): a bare Linear `mods = W_ada · temb + b`
// (M = 1, N = 4H, K = adaln_dim), then folds (1 + scale) into the block's
// norm gains (nw1 = an1 · (1 + scale_msa), nw3 = fn1 · (1 + scale_mlp)).
// Every block reads the SAME temb, so all of them are one weight-streaming
// pass here: the work is reading the packed adaLN weights once (HBM-bound),
// with M <= 4 tokens riding along in registers.
//
// Persistent warps. The n_blocks * N weight rows form one list; warp w of the
// grid owns a contiguous, balanced slice of it and streams it with eight
// 16-byte loads per lane in flight (rows are contiguous in memory, so a warp
// reads whole rows with fully coalesced loads).
//
//  * Row-packed path (a row is 8, 16 or 32 chunks of 16 bytes: K = 256 at
//    w4 / w8 / bf16): one load instruction covers 32 / C whole rows and lane
//    l always reads chunk l % C of its row (its temb values come from shared
//    memory, one 8-byte word per code pair and token, shared by the eight
//    rows in flight). The eight per-instruction partial sums are reduced
//    across the row's C lanes with a transposing butterfly (7 shuffles per
//    token instead of 28).
//  * Generic path (any other K, e.g. the [4H, 3840] shape): a warp per row,
//    lanes striding over the row's chunks, temb from shared memory, a full
//    warp reduction per row.
//
// Quantized weights: a chunk lies inside one 64-wide group, so
//   sum_k (s q_k + b) t_k = s * sum_k q_k t_k + b * sum_k t_k,
// and each code enters as an exact small integer (byte-permute into the float
// 2^23 + q, minus 2^23) in packed fp32-pair FMAs. Every token's sums are
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

// The row's epilogue: bias, the bf16 mods row values of every token, and the
// (1 + scale) folds into the norm gains (chunks 0 and 2 of the 4H outputs).
template <int MT>
__device__ __forceinline__ void write_row(const ModParams& p, const ModBlock& blk, int b, int n,
                                          const float* v) {
  const float bias = bf16_bits_to_f32(blk.bias[n]);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (m >= p.M) break;
    const size_t bm = static_cast<size_t>(b) * p.m_stride + m;
    const __nv_bfloat16 mv = __float2bfloat16_rn(v[m] + bias);
    reinterpret_cast<__nv_bfloat16*>(p.mods)[bm * p.N + n] = mv;
    const float scale1 = 1.0f + __bfloat162float(mv);
    if (p.nw1 != nullptr && blk.an1 != nullptr && n < p.H)
      reinterpret_cast<__nv_bfloat16*>(p.nw1)[bm * p.H + n] =
          __float2bfloat16_rn(bf16_bits_to_f32(blk.an1[n]) * scale1);
    if (p.nw3 != nullptr && blk.fn1 != nullptr && n >= 2 * p.H && n < 3 * p.H)
      reinterpret_cast<__nv_bfloat16*>(p.nw3)[bm * p.H + (n - 2 * p.H)] =
          __float2bfloat16_rn(bf16_bits_to_f32(blk.fn1[n - 2 * p.H]) * scale1);
  }
}

// Balanced contiguous slice [begin, end) of `total` items for warp `w` of `nw`.
__device__ __forceinline__ void warp_slice(long long total, long long w, long long nw,
                                           long long& begin, long long& end) {
  begin = total * w / nw;
  end = total * (w + 1) / nw;
}

// ---- row-packed path: C = 8, 16 or 32 chunks per row ------------------------
// Shared memory: the block table, then this launch's temb as fp32 pairs in
// the order [token][pair of the chunk][chunk] (the lanes of an instruction
// read consecutive 8-byte words), then the per-chunk temb sums [token][chunk].
template <int BITS, int MT, int C>
__global__ void __launch_bounds__(kModThreads) mod_rows_kernel(const __grid_constant__ ModParams p) {
  using F = ModFmt<BITS>;
  constexpr int RI = 32 / C;  // rows per load instruction
  extern __shared__ uint8_t mod_smem[];
  ModBlock* blocks = reinterpret_cast<ModBlock*>(mod_smem);
  const size_t blk_bytes = (static_cast<size_t>(p.n_blocks) * sizeof(ModBlock) + 15) & ~size_t(15);
  uint64_t* t2s = reinterpret_cast<uint64_t*>(mod_smem + blk_bytes);
  float* ts = reinterpret_cast<float*>(t2s + MT * F::kPairs * C);
  for (int i = threadIdx.x; i < p.n_blocks; i += blockDim.x) blocks[i] = p.blocks[i];
  for (int i = threadIdx.x; i < MT * F::kPairs * C; i += blockDim.x) {
    const int m = i / (F::kPairs * C), rem = i % (F::kPairs * C);
    const int q = rem / C, ch = rem % C;
    float a = 0.0f, b = 0.0f;
    if (m < p.M) {
      const uint16_t* t = p.temb + static_cast<size_t>(m) * p.K + ch * F::kPer + 2 * q;
      a = bf16_bits_to_f32(t[0]);
      b = bf16_bits_to_f32(t[1]);
    }
    t2s[i] = f32x2(a, b);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < MT * C; i += blockDim.x) {
    const int m = i / C, ch = i % C;
    float s = 0.0f;
    for (int q = 0; q < F::kPairs; ++q) {
      const uint64_t v = t2s[(m * F::kPairs + q) * C + ch];
      s += f32x2_lo(v);
      s += f32x2_hi(v);
    }
    ts[i] = s;
  }
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int kc = lane % C;      // this lane's chunk of every row it reads
  const int rsub = lane / C;    // its row within an instruction's RI rows
  const int row_bytes = C * 16;
  const uint64_t neg_magic2 = f32x2(-p.code_magic, -p.code_magic);
  float tsum[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) tsum[m] = ts[m * C + kc];
  const int group_of_chunk = BITS == 0 ? 0 : (kc * F::kPer) / 64;

  const long long total_units = static_cast<long long>(p.n_blocks) * p.N / RI;
  const long long nwarps = static_cast<long long>(gridDim.x) * kModWarps;
  const long long gw = static_cast<long long>(blockIdx.x) * kModWarps + (threadIdx.x >> 5);
  long long u_begin, u_end;
  warp_slice(total_units, gw, nwarps, u_begin, u_end);

  for (long long u0 = u_begin; u0 < u_end; u0 += kUnroll) {
    const int nvalid = static_cast<int>(min(static_cast<long long>(kUnroll), u_end - u0));
    const long long row0 = u0 * RI;
    const int b0 = static_cast<int>(row0 / p.N);
    const long long next_block_row = static_cast<long long>(b0 + 1) * p.N;
    uint4 c[kUnroll];
    uint32_t sbw[kUnroll];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      c[j] = make_uint4(0u, 0u, 0u, 0u);
      sbw[j] = 0u;
      if (j < nvalid) {
        const long long r = row0 + j * RI + rsub;
        const int b = r >= next_block_row ? b0 + 1 : b0;
        const int n = static_cast<int>(r - static_cast<long long>(b) * p.N);
        const ModBlock& blk = blocks[b];
        c[j] = ld_global_nc_v4(blk.w + static_cast<size_t>(n) * row_bytes + kc * 16);
        if (BITS != 0) sbw[j] = __ldg(blk.sb + static_cast<size_t>(n) * p.sb_stride + group_of_chunk);
      }
    }
    // per instruction and token: this lane's chunk dot (pairs in order, even
    // and odd weights in two chains), then the group scale and bias
    uint64_t acc[MT][kUnroll];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) acc[m][j] = f32x2(0.0f, 0.0f);
#pragma unroll
    for (int q = 0; q < F::kPairs; ++q) {
      uint64_t tv[MT];
#pragma unroll
      for (int m = 0; m < MT; ++m) tv[m] = t2s[(m * F::kPairs + q) * C + kc];
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) {
        const uint64_t w2 = chunk_pair<BITS>(c[j], q, p.code_xor, neg_magic2);
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m][j] = fma_f32x2(w2, tv[m], acc[m][j]);
      }
    }
    float v[MT][kUnroll];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const float d = f32x2_lo(acc[m][j]) + f32x2_hi(acc[m][j]);
        if constexpr (BITS == 0) {
          v[m][j] = d;
        } else {
          const float sc = bf16_bits_to_f32(sbw[j] & 0xFFFFu);
          const float bi = bf16_bits_to_f32(sbw[j] >> 16);
          v[m][j] = fmaf(sc, d, bi * tsum[m]);
        }
      }
    }
    // Transposing butterfly over the row's C lanes: at offset o the lane
    // with bit o clear keeps the lower half of its values, the other the
    // upper half, each adding its partner's copy; after three halvings a
    // lane holds one instruction's row (index from its bits C/2, C/4, C/8),
    // summed over 8 lanes; plain xor steps finish the sum.
#pragma unroll
    for (int m = 0; m < MT; ++m) {
#pragma unroll
      for (int step = 0; step < 3; ++step) {
        const int o = C >> (step + 1);
        const int half = kUnroll >> (step + 1);
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
          const float send = upper ? v[m][i] : v[m][i + half];
          const float keep = upper ? v[m][i + half] : v[m][i];
          v[m][i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, o);
        }
      }
#pragma unroll
      for (int o = C >> 4; o > 0; o >>= 1) v[m][0] += __shfl_xor_sync(0xFFFFFFFFu, v[m][0], o);
    }
    const int jrow = ((lane & (C >> 1)) ? 4 : 0) + ((lane & (C >> 2)) ? 2 : 0) +
                     ((lane & (C >> 3)) ? 1 : 0);
    const bool writer = (kc & ((C >> 3) - 1)) == 0;
    if (writer && jrow < nvalid) {
      const long long r = row0 + jrow * RI + rsub;
      const int b = r >= next_block_row ? b0 + 1 : b0;
      const int n = static_cast<int>(r - static_cast<long long>(b) * p.N);
      float out[MT];
#pragma unroll
      for (int m = 0; m < MT; ++m) out[m] = v[m][0];
      write_row<MT>(p, blocks[b], b, n, out);
    }
  }
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
  for (long long r = r_begin; r < r_end; ++r) {
    const int b = static_cast<int>(r / p.N);
    const int n = static_cast<int>(r - static_cast<long long>(b) * p.N);
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
cudaError_t launch_mod_t(const ModParams& p, cudaStream_t stream) {
  const int row_bytes = BITS == 0 ? p.K * 2 : p.K * BITS / 8;
  const int C = row_bytes / 16;
  const size_t blk_bytes = (static_cast<size_t>(p.n_blocks) * sizeof(ModBlock) + 15) & ~size_t(15);
  const long long rows = static_cast<long long>(p.n_blocks) * p.N;
  if (C == 8 || C == 16 || C == 32) {
    const int ri = 32 / C;
    // a group of eight instructions then spans at most one block boundary
    if (p.N % ri == 0 && p.N >= kUnroll * ri) {
      const long long work = (rows / ri + kUnroll - 1) / kUnroll;  // warps with a full group
      const size_t smem = blk_bytes + static_cast<size_t>(MT) * ModFmt<BITS>::kPairs * C * 8 +
                          static_cast<size_t>(MT) * C * 4;
      static std::atomic<int> cache8[64], cache16[64], cache32[64];
      if (C == 8) return launch_persistent(mod_rows_kernel<BITS, MT, 8>, p, smem, work, cache8, stream);
      if (C == 16) return launch_persistent(mod_rows_kernel<BITS, MT, 16>, p, smem, work, cache16, stream);
      return launch_persistent(mod_rows_kernel<BITS, MT, 32>, p, smem, work, cache32, stream);
    }
  }
  constexpr int Q = ModFmt<BITS>::kPer / 4;
  const size_t smem = blk_bytes + static_cast<size_t>(MT) * Q * C * 16 + static_cast<size_t>(MT) * C * 4;
  static std::atomic<int> cachew[64];
  return launch_persistent(mod_warp_kernel<BITS, MT>, p, smem, rows, cachew, stream);
}

// Token count rounded up to 1, 2 or 4: registers scale with it.
template <int BITS>
cudaError_t launch_mod_bits(const ModParams& p, cudaStream_t stream) {
  if (p.M == 1) return launch_mod_t<BITS, 1>(p, stream);
  if (p.M == 2) return launch_mod_t<BITS, 2>(p, stream);
  return launch_mod_t<BITS, 4>(p, stream);
}

}  // namespace

cudaError_t launch_mod(const ModParams& p, cudaStream_t stream) {
  const int row_bytes = p.bits == 0 ? p.K * 2 : p.K * p.bits / 8;
  if (row_bytes % 16 != 0 || p.M < 1 || p.M > kModMaxTok || p.m_stride < p.M)
    return cudaErrorInvalidValue;
  if (p.bits != 0 && p.K % 64 != 0) return cudaErrorInvalidValue;
  if (p.bits == 8) return launch_mod_bits<8>(p, stream);
  if (p.bits == 4) return launch_mod_bits<4>(p, stream);
  return launch_mod_bits<0>(p, stream);
}

}  // namespace mp
