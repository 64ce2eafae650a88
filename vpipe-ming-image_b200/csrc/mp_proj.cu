// The fused projection kernel for sm_100a:
//
//   y[M, N] = x[M, K] · deq(W)[N, K]^T  +  T[M, R] · Bstack[N, R]^T
//
// where deq(W) is the packed w8/w4 affine group-64 weight (or a dense bf16
// weight), and T = strength-scaled x · Astack^T is the stacked LoRA
// rank-space intermediate (produced by the same kernel in dense mode with the
// epilogue scaling switched on). This is the arithmetic of the reference's
// `lin` (src/ming-dit.cc:1763-1771): `lin_base` (:1721-1758) followed by
// `lora::Applier::apply` for every live slot — here as ONE pass over K, with
// the adapters appended as extra K tiles of the same accumulation.
//
// Layout (swap-AB): the MMA's M dimension is 128 output features, its N
// dimension is up to 256 tokens. Per 64-wide K stage:
//   * warp 0 (one thread) issues TMA loads of the activation tile (SW128) and
//     the weight tile (codes with SW64/SW32, or bf16 with SW128);
//   * warps 2-5 dequantize the codes tile: thread r owns output feature r,
//     computes w = scale·q + bias in fp32, rounds to bf16 and stores its row
//     into TMEM (tcgen05.st) — the MMA reads A straight from TMEM, so the
//     dequantized weight never touches shared or global memory;
//   * warp 1 (one thread) issues tcgen05.mma: TMEM-A x SMEM-B for packed
//     tiles, SMEM x SMEM for dense and LoRA tiles, accumulating f32 in TMEM;
//   * after the last K tile, warps 2-5 read the accumulator (tcgen05.ld) and
//     write bf16 rows of y.
#include <cuda_runtime.h>

#include "mp_device.cuh"
#include "mp_kernels.h"

namespace mp {

namespace {

enum : uint32_t {
  kSiteProducerEmpty = 0x100u,
  kSiteMmaFull = 0x200u,
  kSiteMmaDeq = 0x300u,
  kSiteDeqFull = 0x400u,
  kSiteEpilogue = 0x500u,
  kSiteDrain = 0x600u,
};

// 4 packed 8-bit codes -> 4 bf16 weights in two bf16x2 words.
__device__ __forceinline__ void deq8_word(uint32_t w, float sc, float bi, float magic,
                                          uint32_t& p0, uint32_t& p1) {
  const float q0 = __uint_as_float(__byte_perm(w, 0x4Bu, 0x4550u)) - magic;
  const float q1 = __uint_as_float(__byte_perm(w, 0x4Bu, 0x4551u)) - magic;
  const float q2 = __uint_as_float(__byte_perm(w, 0x4Bu, 0x4552u)) - magic;
  const float q3 = __uint_as_float(__byte_perm(w, 0x4Bu, 0x4553u)) - magic;
  p0 = pack_bf16x2(fmaf(q0, sc, bi), fmaf(q1, sc, bi));
  p1 = pack_bf16x2(fmaf(q2, sc, bi), fmaf(q3, sc, bi));
}

// 8 packed 4-bit codes (code j at bits [4j, 4j+4)) -> 8 bf16 weights.
__device__ __forceinline__ void deq4_word(uint32_t w, float sc, float bi, float magic,
                                          uint32_t* p) {
  const uint32_t ev = w & 0x0F0F0F0Fu;          // codes 0, 2, 4, 6
  const uint32_t od = (w >> 4) & 0x0F0F0F0Fu;   // codes 1, 3, 5, 7
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t sel = 0x4550u | static_cast<uint32_t>(b);
    const float qe = __uint_as_float(__byte_perm(ev, 0x4Bu, sel)) - magic;
    const float qo = __uint_as_float(__byte_perm(od, 0x4Bu, sel)) - magic;
    p[b] = pack_bf16x2(fmaf(qe, sc, bi), fmaf(qo, sc, bi));
  }
}

__device__ __forceinline__ uint32_t pick4(const uint4& v, int i) {
  uint32_t r = v.x;
  r = (i == 1) ? v.y : r;
  r = (i == 2) ? v.z : r;
  r = (i == 3) ? v.w : r;
  return r;
}

struct Smem {
  uint8_t* tiles;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* afull;
  uint64_t* tfull;
  uint64_t* drain;
  uint32_t* tmem_slot;
  volatile uint32_t* abort;
};

__device__ __forceinline__ Smem carve(uint8_t* raw) {
  Smem s;
  const uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 1023u) & ~uintptr_t(1023u);
  s.tiles = reinterpret_cast<uint8_t*>(base);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s.tiles + kStages * kStageBytes);
  s.full = bars;
  s.empty = bars + kStages;
  s.afull = bars + 2 * kStages;
  s.tfull = bars + 3 * kStages;
  s.drain = s.tfull + 1;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.drain + 1);
  s.abort = s.tmem_slot + 1;
  return s;
}

__device__ void producer(const ProjParams& p, const Smem& sm, int n0, int m0, int base_kt,
                         int total_kt) {
  const bool quant = p.bits != 0;
  const uint32_t xbytes = static_cast<uint32_t>(p.n_tok) * 128u;
  const uint32_t wbytes_base =
      quant ? static_cast<uint32_t>(kBlockN * kBlockK * p.bits / 8) : uint32_t(kWStageBytes);
  int issued = 0;
  for (int kt = 0; kt < total_kt; ++kt) {
    const int s = kt % kStages;
    const uint32_t ph = static_cast<uint32_t>(kt / kStages) & 1u;
    if (kt >= kStages &&
        !mbar_wait(smem_u32(&sm.empty[s]), ph ^ 1u, sm.abort, kSiteProducerEmpty | s,
                   p.wait_limit_ns))
      break;
    uint8_t* xb = sm.tiles + s * kStageBytes;
    uint8_t* wb = xb + kXStageBytes;
    const uint32_t bar = smem_u32(&sm.full[s]);
    if (kt < base_kt) {
      mbar_arrive_expect_tx(bar, xbytes + wbytes_base);
      tma_load_2d(smem_u32(xb), &p.tm_x, bar, kt * kBlockK, m0);
      tma_load_2d(smem_u32(wb), &p.tm_w, bar, quant ? kt * kBlockK * p.bits / 8 : kt * kBlockK,
                  n0);
    } else {
      const int j = kt - base_kt;
      mbar_arrive_expect_tx(bar, xbytes + uint32_t(kWStageBytes));
      tma_load_2d(smem_u32(xb), &p.tm_t, bar, j * kBlockK, m0);
      tma_load_2d(smem_u32(wb), &p.tm_b, bar, j * kBlockK, n0);
    }
    issued = kt + 1;
  }
  if (*sm.abort != 0u) {
    // Unwind: wait (bounded) until every load this thread issued has landed,
    // so no copy writes into shared memory after the CTA has gone.
    for (int kt = issued - kStages < 0 ? 0 : issued - kStages; kt < issued; ++kt) {
      const int s = kt % kStages;
      const uint32_t ph = static_cast<uint32_t>(kt / kStages) & 1u;
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(smem_u32(&sm.full[s]), ph)) {
        if (global_timer_ns() - t0 > p.wait_limit_ns) break;
      }
    }
  }
}

__device__ void mma_issuer(const ProjParams& p, const Smem& sm, uint32_t tmem, int base_kt,
                           int total_kt) {
  const bool quant = p.bits != 0;
  const uint32_t idesc = make_idesc_bf16(kBlockN, static_cast<uint32_t>(p.n_tok));
  uint32_t acc = 0;
  for (int kt = 0; kt < total_kt; ++kt) {
    const int s = kt % kStages;
    const uint32_t ph = static_cast<uint32_t>(kt / kStages) & 1u;
    if (!mbar_wait(smem_u32(&sm.full[s]), ph, sm.abort, kSiteMmaFull | s, p.wait_limit_ns)) break;
    const bool from_tmem = quant && kt < base_kt;
    if (from_tmem &&
        !mbar_wait(smem_u32(&sm.afull[s]), ph, sm.abort, kSiteMmaDeq | s, p.wait_limit_ns))
      break;
    tc_fence_after();
    const uint32_t xaddr = smem_u32(sm.tiles + s * kStageBytes);
    const uint32_t waddr = xaddr + kXStageBytes;
#pragma unroll
    for (int kk = 0; kk < kBlockK / 16; ++kk) {
      const uint64_t bdesc = make_sdesc_sw128(xaddr + kk * 32);
      if (from_tmem) {
        umma_ts(tmem + kAccCol, tmem + kACol + s * 32 + kk * 8, bdesc, idesc, acc);
      } else {
        umma_ss(tmem + kAccCol, make_sdesc_sw128(waddr + kk * 32), bdesc, idesc, acc);
      }
      acc = 1;
    }
    umma_commit(smem_u32(&sm.empty[s]));
  }
  if (*sm.abort == 0u) umma_commit(smem_u32(sm.tfull));
  // Drain: nothing this thread issued may still be reading TMEM or shared
  // memory when the CTA frees them.
  umma_commit(smem_u32(sm.drain));
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(smem_u32(sm.drain), 0)) {
    if (global_timer_ns() - t0 > p.wait_limit_ns) {
      atomicCAS(const_cast<uint32_t*>(sm.abort), 0u, kSiteDrain);
      break;
    }
  }
}

// Warps 2-5: thread (warp % 4, lane) owns output feature row r of the tile.
__device__ void dequantizer(const ProjParams& p, const Smem& sm, uint32_t tmem, int n0,
                            int base_kt) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q = warp & 3;
  const int r = q * 32 + lane;
  const int n = n0 + r;
  const bool row_ok = n < p.N;
  const uint32_t* sbrow = p.sb + static_cast<size_t>(row_ok ? n : 0) * p.sb_stride;
  const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
  uint4 sbv = make_uint4(0, 0, 0, 0);
  for (int kt = 0; kt < base_kt; ++kt) {
    const int s = kt % kStages;
    const uint32_t ph = static_cast<uint32_t>(kt / kStages) & 1u;
    if ((kt & 3) == 0) sbv = row_ok ? ld_global_nc_v4(sbrow + kt) : make_uint4(0, 0, 0, 0);
    const uint32_t sbw = pick4(sbv, kt & 3);
    const float sc = bf16_bits_to_f32(sbw & 0xFFFFu);
    const float bi = bf16_bits_to_f32(sbw >> 16);
    if (!mbar_wait(smem_u32(&sm.full[s]), ph, sm.abort, kSiteDeqFull | s, p.wait_limit_ns)) break;
    const uint32_t wb = smem_u32(sm.tiles + s * kStageBytes + kXStageBytes);
    uint32_t packed[32];
    if (p.bits == 8) {
      const uint32_t sw = static_cast<uint32_t>((r >> 1) & 3);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 c = ld_shared_v4(wb + r * 64 + ((static_cast<uint32_t>(j) ^ sw) << 4));
        deq8_word(c.x ^ p.code_xor, sc, bi, p.code_magic, packed[8 * j + 0], packed[8 * j + 1]);
        deq8_word(c.y ^ p.code_xor, sc, bi, p.code_magic, packed[8 * j + 2], packed[8 * j + 3]);
        deq8_word(c.z ^ p.code_xor, sc, bi, p.code_magic, packed[8 * j + 4], packed[8 * j + 5]);
        deq8_word(c.w ^ p.code_xor, sc, bi, p.code_magic, packed[8 * j + 6], packed[8 * j + 7]);
      }
    } else {
      const uint32_t sw = static_cast<uint32_t>((r >> 2) & 1);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint4 c = ld_shared_v4(wb + r * 32 + ((static_cast<uint32_t>(j) ^ sw) << 4));
        deq4_word(c.x, sc, bi, p.code_magic, &packed[16 * j + 0]);
        deq4_word(c.y, sc, bi, p.code_magic, &packed[16 * j + 4]);
        deq4_word(c.z, sc, bi, p.code_magic, &packed[16 * j + 8]);
        deq4_word(c.w, sc, bi, p.code_magic, &packed[16 * j + 12]);
      }
    }
    MP_TMEM_ST_32X32B_X32(tmem + lane_base + kACol + s * 32, packed);
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(smem_u32(&sm.afull[s]));
  }
}

__device__ __forceinline__ float epilogue_scale(const EpilogueScale& es, int t, int slot) {
  int g = 0;
  while (g + 1 < es.n_seg && t >= es.seg_start[g + 1]) ++g;
  return es.seg_scale[g][slot];
}

__device__ void epilogue(const ProjParams& p, const Smem& sm, uint32_t tmem, int n0, int m0) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q = warp & 3;
  const int r = q * 32 + lane;
  const int f = n0 + r;
  const bool ok = mbar_wait(smem_u32(sm.tfull), 0, sm.abort, kSiteEpilogue, p.wait_limit_ns);
  if (!ok) return;
  tc_fence_after();
  int slot = -1;
  if (p.scale.enabled) {
    for (int i = 0; i < p.scale.n_ranges; ++i)
      if (f >= p.scale.range_start[i] && f < p.scale.range_start[i + 1]) slot = p.scale.range_slot[i];
  }
  __nv_bfloat16* y = static_cast<__nv_bfloat16*>(p.y);
  const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
  for (int c = 0; c < p.n_tok / 32; ++c) {
    uint32_t v[32];
    MP_TMEM_LD_32X32B_X32(tmem + lane_base + kAccCol + c * 32, v);
    tmem_wait_ld();
    const int t0 = m0 + c * 32;
    if (f < p.N) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int t = t0 + j;
        if (t < p.M) {
          float val = __uint_as_float(v[j]);
          if (p.scale.enabled) val = slot >= 0 ? val * epilogue_scale(p.scale, t, slot) : 0.0f;
          y[static_cast<size_t>(t) * p.ldy + f] = __float2bfloat16_rn(val);
        }
      }
    }
  }
}

}  // namespace

__global__ void __launch_bounds__(kProjThreads, 1) proj_kernel(const __grid_constant__ ProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  const Smem sm = carve(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBlockN;
  const int m0 = blockIdx.y * p.n_tok;
  const int base_kt = p.K / kBlockK;
  const int total_kt = base_kt + p.lora_ktiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&sm.full[s]), 1);
      mbar_init(smem_u32(&sm.empty[s]), 1);
      mbar_init(smem_u32(&sm.afull[s]), 128);
    }
    mbar_init(smem_u32(sm.tfull), 1);
    mbar_init(smem_u32(sm.drain), 1);
    *sm.abort = 0u;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&p.tm_x);
    tma_prefetch_map(&p.tm_w);
    if (p.lora_ktiles > 0) {
      tma_prefetch_map(&p.tm_t);
      tma_prefetch_map(&p.tm_b);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(sm.tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_slot;

  if (warp == 0) {
    if (lane == 0) producer(p, sm, n0, m0, base_kt, total_kt);
  } else if (warp == 1) {
    if (lane == 0) mma_issuer(p, sm, tmem, base_kt, total_kt);
  } else {
    if (p.bits != 0) dequantizer(p, sm, tmem, n0, base_kt);
    epilogue(p, sm, tmem, n0, m0);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
  if (threadIdx.x == 0 && *sm.abort != 0u) atomicOr(p.err, kErrTimeout);
}

cudaError_t launch_proj(const ProjParams& p, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kProjSmemBytes));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid((p.N + kBlockN - 1) / kBlockN, (p.M + p.n_tok - 1) / p.n_tok);
  proj_kernel<<<grid, kProjThreads, kProjSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace mp
