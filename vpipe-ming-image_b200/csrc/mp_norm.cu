// The sandwich-norm residual step of a DiT block as one pass over the rows:
//
//   s   = bf16(o * rsqrt(mean(o^2) + eps) * o_gain)          (o given)
//   x   = bf16(x + tanh(gate) * s)  (gate given)  or  bf16(x + s)
//   nrm = bf16(x * rsqrt(mean(x^2) + eps) * nrm_gain)        (nrm given)
//
// The reference runs these as three passes after to_out and after w2: rms of
// the sub-layer output in place, gated_residual_tanh (or the plain residual)
// into the joint stream, rms of the joint stream into the next sub-layer's
// input (src/ming-dit.cc:2096-2101, :2256-2261; gated_residual_tanh_v4_f16,
// src/metal/ming_ops.metal:55-93). The row norm spans all output features of
// the projection (every CTA pair of its launch), so it runs here, after the
// projection, rather than in the projection's epilogue.
//
// Memory-bound: per row it reads o and x and writes x and nrm once (16-byte
// accesses). A CTA of 256 threads walks rows blockIdx.x, + gridDim.x, ...
// (a few CTAs per SM), with the next row's x and o loads in flight while
// the current row is reduced and stored; tanh(gate) is tabulated once per
// CTA in shared memory. The arithmetic runs on packed fp32 pairs (each
// product and sum rounded once, as the scalar sequence). Each row's two sums
// of squares are reduced in a fixed order (even and odd elements as one
// packed FMA chain per thread, warp xor tree, warps in order), so results do
// not depend on timing.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "mp_device.cuh"
#include "mp_kernels.h"

namespace mp {

namespace {

constexpr int kNormThreads = 256;
constexpr int kNormWarps = kNormThreads / 32;
constexpr int kNormCtasPerSm = 4;

// bf16x2 word -> packed fp32 pair (low half from the low bf16)
__device__ __forceinline__ uint64_t unpack2(uint32_t w) {
  return (static_cast<uint64_t>(w & 0xFFFF0000u) << 32) | static_cast<uint64_t>(w << 16);
}

// Sum over the CTA, in a fixed order. `red` alternates between two buffers
// call by call: the barrier of the next call orders this call's reads
// before the buffer is written again, so one barrier per call suffices.
__device__ __forceinline__ float cta_sum(float v, float (*red)[kNormWarps], int& parity) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
  float* buf = red[parity];
  parity ^= 1;
  if ((threadIdx.x & 31) == 0) buf[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = buf[0];
#pragma unroll
  for (int w = 1; w < kNormWarps; ++w) t += buf[w];
  return t;
}

// Sum of squares of this thread's chunks (two chains, even and odd elements,
// as one packed fp32 pair).
template <int CH>
__device__ __forceinline__ float sum_squares(const uint4 (&v)[CH], int chunks) {
  uint64_t s2 = 0ull;
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = static_cast<int>(threadIdx.x) + i * kNormThreads;
    if (c < chunks) {
      const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint64_t a = unpack2(w[e]);
        s2 = fma_f32x2(a, a, s2);
      }
    }
  }
  return f32x2_lo(s2) + f32x2_hi(s2);
}

template <int CH>
__device__ __forceinline__ void load_row(const RmsResidualParams& p, int r, int chunks,
                                         uint4 (&xv)[CH], uint4 (&ov)[CH]) {
  const uint16_t* xrow = p.x + static_cast<size_t>(r) * p.ldx;
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = static_cast<int>(threadIdx.x) + i * kNormThreads;
    if (c < chunks) xv[i] = *reinterpret_cast<const uint4*>(xrow + 8 * c);
  }
  if (p.o != nullptr) {
    const uint16_t* orow = p.o + static_cast<size_t>(r) * p.ldo;
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int c = static_cast<int>(threadIdx.x) + i * kNormThreads;
      if (c < chunks) ov[i] = *reinterpret_cast<const uint4*>(orow + 8 * c);
    }
  }
}

template <int CH>
__device__ __forceinline__ void process_row(const RmsResidualParams& p, int r, int chunks,
                                            float inv_h, const float* tgate,
                                            float (*red)[kNormWarps], int& parity,
                                            uint4 (&xv)[CH], const uint4 (&ov)[CH]) {
  if (p.o != nullptr) {
    const float ro =
        rsqrtf(__fadd_rn(__fmul_rn(cta_sum(sum_squares<CH>(ov, chunks), red, parity), inv_h), p.eps));
    const uint64_t ro2 = f32x2(ro, ro);
    uint16_t* xrow = p.x + static_cast<size_t>(r) * p.ldx;
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int c = static_cast<int>(threadIdx.x) + i * kNormThreads;
      if (c >= chunks) continue;
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(p.o_gain) + c);
      const uint32_t ow[4] = {ov[i].x, ov[i].y, ov[i].z, ov[i].w};
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
      uint32_t xw[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        // s = bf16((o * ro) * gain): the sub-layer output's RMSNorm
        const uint32_t sw = f32x2_to_bf16x2(mul_f32x2(mul_f32x2(unpack2(ow[e]), ro2), unpack2(gw[e])));
        uint64_t s2 = unpack2(sw);
        if (p.gate != nullptr) {
          const float2 tg = *reinterpret_cast<const float2*>(tgate + 8 * c + 2 * e);
          s2 = mul_f32x2(f32x2(tg.x, tg.y), s2);
        }
        xw[e] = f32x2_to_bf16x2(add_f32x2(unpack2(xw[e]), s2));
      }
      xv[i] = make_uint4(xw[0], xw[1], xw[2], xw[3]);
      *reinterpret_cast<uint4*>(xrow + 8 * c) = xv[i];
    }
  }
  if (p.nrm != nullptr) {
    const float rx =
        rsqrtf(__fadd_rn(__fmul_rn(cta_sum(sum_squares<CH>(xv, chunks), red, parity), inv_h), p.eps));
    const uint64_t rx2 = f32x2(rx, rx);
    uint16_t* nrow = p.nrm + static_cast<size_t>(r) * p.ldn;
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int c = static_cast<int>(threadIdx.x) + i * kNormThreads;
      if (c >= chunks) continue;
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(p.nrm_gain) + c);
      const uint32_t xw[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
      uint32_t nw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        nw[e] = f32x2_to_bf16x2(mul_f32x2(mul_f32x2(unpack2(xw[e]), rx2), unpack2(gw[e])));
      *reinterpret_cast<uint4*>(nrow + 8 * c) = make_uint4(nw[0], nw[1], nw[2], nw[3]);
    }
  }
}

// CH = 16-byte chunks per thread and row (H / 8 / 256, rounded up).
template <int CH>
__global__ void __launch_bounds__(kNormThreads) rms_residual_kernel(const RmsResidualParams p) {
  extern __shared__ float tgate[];  // [H] tanh(gate) (gated calls)
  __shared__ float red[2][kNormWarps];
  const int chunks = p.H / 8;
  const float inv_h = 1.0f / static_cast<float>(p.H);  // mean = sum * (1 / H)
  if (p.gate != nullptr) {
    for (int i = threadIdx.x; i < p.H; i += kNormThreads)
      tgate[i] = tanhf(__uint_as_float(static_cast<uint32_t>(p.gate[i]) << 16));
    __syncthreads();
  }
  int parity = 0;
  const int step = static_cast<int>(gridDim.x);
  int r = static_cast<int>(blockIdx.x);
  if (r >= p.M) return;
  uint4 xa[CH], oa[CH], xb[CH], ob[CH];
  load_row<CH>(p, r, chunks, xa, oa);
  // two rows per iteration, so the register buffers keep fixed names
#pragma unroll 1
  for (; r < p.M; r += 2 * step) {
    if (r + step < p.M) load_row<CH>(p, r + step, chunks, xb, ob);
    process_row<CH>(p, r, chunks, inv_h, tgate, red, parity, xa, oa);
    if (r + step >= p.M) break;
    if (r + 2 * step < p.M) load_row<CH>(p, r + 2 * step, chunks, xa, oa);
    process_row<CH>(p, r + step, chunks, inv_h, tgate, red, parity, xb, ob);
  }
}

template <int CH>
cudaError_t launch_ch(const RmsResidualParams& p, cudaStream_t stream) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int blocks = p.M < sms * kNormCtasPerSm ? p.M : sms * kNormCtasPerSm;
  const size_t smem = p.gate != nullptr ? static_cast<size_t>(p.H) * sizeof(float) : 0;
  rms_residual_kernel<CH><<<blocks, kNormThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_rms_residual(const RmsResidualParams& p, cudaStream_t stream) {
  const int ch = (p.H / 8 + kNormThreads - 1) / kNormThreads;
  static_assert(kNormMaxH / 8 / kNormThreads == 4, "chunk counts dispatched below");
  switch (ch) {
    case 1: return launch_ch<1>(p, stream);
    case 2: return launch_ch<2>(p, stream);
    case 3: return launch_ch<3>(p, stream);
    default: return launch_ch<4>(p, stream);
  }
}

}  // namespace mp
