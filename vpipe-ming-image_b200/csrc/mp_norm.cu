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
// HBM-bound: per row it reads o and x and writes x and nrm once (16-byte
// accesses). A CTA of 256 threads takes kRowsPerCta rows; tanh(gate) is
// tabulated once per CTA in shared memory. Each row's two sums of squares are
// reduced in a fixed order (per-thread sequential, warp xor tree, warps in
// order), so results do not depend on timing.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "mp_kernels.h"

namespace mp {

namespace {

constexpr int kNormThreads = 256;
constexpr int kNormWarps = kNormThreads / 32;
constexpr int kRowsPerCta = 4;
constexpr int kMaxChunks = kNormMaxH / 8 / kNormThreads;  // 16-byte chunks per thread

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Sum over the CTA, in a fixed order; `red` holds kNormWarps floats and is
// free again when this returns (the trailing barrier).
__device__ __forceinline__ float cta_sum(float v, float* red) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int w = 1; w < kNormWarps; ++w) t += red[w];
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(kNormThreads) rms_residual_kernel(const RmsResidualParams p) {
  extern __shared__ float tgate[];  // [H] tanh(gate) (gated calls)
  __shared__ float red[kNormWarps];
  const int chunks = p.H / 8;
  const float inv_h = 1.0f / static_cast<float>(p.H);  // mean = sum * (1 / H)
  if (p.gate != nullptr) {
    for (int i = threadIdx.x; i < p.H; i += kNormThreads)
      tgate[i] = tanhf(__uint_as_float(static_cast<uint32_t>(p.gate[i]) << 16));
    __syncthreads();
  }
  const int row_end = min(p.M, (static_cast<int>(blockIdx.x) + 1) * kRowsPerCta);
  for (int r = static_cast<int>(blockIdx.x) * kRowsPerCta; r < row_end; ++r) {
    uint16_t* xrow = p.x + static_cast<size_t>(r) * p.ldx;
    uint4 xv[kMaxChunks];
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      const int c = static_cast<int>(threadIdx.x) + i * kNormThreads;
      if (c < chunks) xv[i] = *reinterpret_cast<const uint4*>(xrow + 8 * c);
    }
    if (p.o != nullptr) {
      const uint16_t* orow = p.o + static_cast<size_t>(r) * p.ldo;
      uint4 ov[kMaxChunks];
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < kMaxChunks; ++i) {
        const int c = static_cast<int>(threadIdx.x) + i * kNormThreads;
        if (c < chunks) {
          ov[i] = *reinterpret_cast<const uint4*>(orow + 8 * c);
          const uint32_t w[4] = {ov[i].x, ov[i].y, ov[i].z, ov[i].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            ss = __fadd_rn(ss, __fmul_rn(bf16lo(w[e]), bf16lo(w[e])));
            ss = __fadd_rn(ss, __fmul_rn(bf16hi(w[e]), bf16hi(w[e])));
          }
        }
      }
      const float ro = rsqrtf(__fadd_rn(__fmul_rn(cta_sum(ss, red), inv_h), p.eps));
#pragma unroll
      for (int i = 0; i < kMaxChunks; ++i) {
        const int c = static_cast<int>(threadIdx.x) + i * kNormThreads;
        if (c >= chunks) continue;
        const uint4 gv = __ldg(reinterpret_cast<const uint4*>(p.o_gain) + c);
        const uint32_t ow[4] = {ov[i].x, ov[i].y, ov[i].z, ov[i].w};
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
        uint32_t xw[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int f = 8 * c + 2 * e;
          // s = bf16((o * ro) * gain): the sub-layer output's RMSNorm
          const uint32_t sw = pack2(__fmul_rn(__fmul_rn(bf16lo(ow[e]), ro), bf16lo(gw[e])),
                                    __fmul_rn(__fmul_rn(bf16hi(ow[e]), ro), bf16hi(gw[e])));
          float s0 = bf16lo(sw), s1 = bf16hi(sw);
          if (p.gate != nullptr) {
            s0 = __fmul_rn(tgate[f], s0);
            s1 = __fmul_rn(tgate[f + 1], s1);
          }
          xw[e] = pack2(__fadd_rn(bf16lo(xw[e]), s0), __fadd_rn(bf16hi(xw[e]), s1));
        }
        xv[i] = make_uint4(xw[0], xw[1], xw[2], xw[3]);
        *reinterpret_cast<uint4*>(xrow + 8 * c) = xv[i];
      }
    }
    if (p.nrm != nullptr) {
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < kMaxChunks; ++i) {
        const int c = static_cast<int>(threadIdx.x) + i * kNormThreads;
        if (c < chunks) {
          const uint32_t w[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            ss = __fadd_rn(ss, __fmul_rn(bf16lo(w[e]), bf16lo(w[e])));
            ss = __fadd_rn(ss, __fmul_rn(bf16hi(w[e]), bf16hi(w[e])));
          }
        }
      }
      const float rx = rsqrtf(__fadd_rn(__fmul_rn(cta_sum(ss, red), inv_h), p.eps));
      uint16_t* nrow = p.nrm + static_cast<size_t>(r) * p.ldn;
#pragma unroll
      for (int i = 0; i < kMaxChunks; ++i) {
        const int c = static_cast<int>(threadIdx.x) + i * kNormThreads;
        if (c >= chunks) continue;
        const uint4 gv = __ldg(reinterpret_cast<const uint4*>(p.nrm_gain) + c);
        const uint32_t xw[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
        uint32_t nw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          nw[e] = pack2(__fmul_rn(__fmul_rn(bf16lo(xw[e]), rx), bf16lo(gw[e])),
                        __fmul_rn(__fmul_rn(bf16hi(xw[e]), rx), bf16hi(gw[e])));
        *reinterpret_cast<uint4*>(nrow + 8 * c) = make_uint4(nw[0], nw[1], nw[2], nw[3]);
      }
    }
  }
}

}  // namespace

cudaError_t launch_rms_residual(const RmsResidualParams& p, cudaStream_t stream) {
  const unsigned blocks = static_cast<unsigned>((p.M + kRowsPerCta - 1) / kRowsPerCta);
  const size_t smem = p.gate != nullptr ? static_cast<size_t>(p.H) * sizeof(float) : 0;
  rms_residual_kernel<<<blocks, kNormThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace mp
