// norms.cu -- fused LayerNorm / RMSNorm forward and backward (bf16 I/O, fp32 math).
//
// Forward: one warp per row; the row stays in registers (16-byte vector loads)
// so x is read once and y written once.  Backward: one warp per row for dx
// (optionally adding the residual-stream gradient in the same pass), with the
// parameter gradients reduced over the block's rows in shared memory and then
// accumulated into fp32 gradient buffers with one atomic per column per block.
//
// Replaces nn.LayerNorm (reference models/tiny_transformer.py:36,39,55).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "mt_api.h"
#include "sm100.cuh"

namespace mt {
namespace {

constexpr int kWarps = 8;          // rows processed concurrently per block
constexpr int kMaxVec = 16;        // 16 x 8 bf16 per lane -> d <= 4096 held in registers

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* f) {
  uint4 q = *reinterpret_cast<const uint4*>(p);
  uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 t = unpack_bf16x2(w[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

__device__ __forceinline__ void unpack8(uint4 q, float* f) {
  uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 t = unpack_bf16x2(w[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* f) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                            pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
}

// RMS = true: RMSNorm (no mean, no beta).  NV = 16-byte vectors per lane.
template <bool RMS, int NV>
__global__ void __launch_bounds__(kWarps * 32)
    norm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ gamma,
                    const __nv_bfloat16* __restrict__ beta, __nv_bfloat16* __restrict__ y,
                    float* __restrict__ mean_out, float* __restrict__ rstd_out, int T, int d, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarps + warp;
  if (row >= T) return;
  const int nvec = d >> 3;  // d % 8 == 0 checked by the launcher
  const __nv_bfloat16* xr = x + (long)row * d;
  float v[NV][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      load8(xr + c * 8, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[i][j];
    }
  }
  float mean = 0.f;
  if constexpr (!RMS) mean = warp_sum(s) / d;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float t = v[i][j] - mean;
        ss += t * t;
      }
    }
  }
  const float var = warp_sum(ss) / d;
  const float rstd = rsqrtf(var + eps);
  __nv_bfloat16* yr = y + (long)row * d;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      float g[8], b[8], o[8];
      load8(gamma + c * 8, g);
      if constexpr (!RMS) load8(beta + c * 8, b);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (v[i][j] - mean) * rstd * g[j] + (RMS ? 0.f : b[j]);
      store8(yr + c * 8, o);
    }
  }
  if (lane == 0) {
    if constexpr (!RMS) mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// Backward.  One warp per row: s1 = sum(dy*g), s2 = sum(dy*g*xhat) by warp
// shuffles, then dx = rstd*(dy*g - s1/d - xhat*s2/d) (+ the residual-stream
// gradient).  Parameter-gradient partials (dgamma = sum dy*xhat, dbeta = sum dy)
// accumulate per warp in shared memory with no atomics: a lane owns the same
// columns of every row, stored transposed ([vec][j][lane]) so each access is
// bank-conflict free.  At the end the block sums its warps' partials and adds
// one value per column into the fp32 gradient buffers.
//
// CACHE: the whole row (NV 16-byte vectors of x and of dy per lane) stays in
// registers between the two phases; otherwise phase two re-reads it (L1 hits).
// All loads of a phase are issued before the first use to keep many 16-byte
// requests in flight per warp.
template <bool RMS, int NV, bool CACHE>
__global__ void __launch_bounds__(kWarps * 32, 2)
    norm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                    const __nv_bfloat16* __restrict__ gamma, const float* __restrict__ mean_in,
                    const float* __restrict__ rstd_in, const __nv_bfloat16* __restrict__ dres,
                    __nv_bfloat16* __restrict__ dx, float* __restrict__ dgamma, float* __restrict__ dbeta,
                    int T, int d, int rows_per_block) {
  constexpr int NACC = RMS ? 1 : 2;
  extern __shared__ float red[];  // [warps][NACC][NV*8][32]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int nvec = d >> 3;
  constexpr int SLOT = NV * 8 * 32;  // floats per accumulator per warp
  float* acc_g = red + warp * NACC * SLOT;
  float* acc_b = acc_g + SLOT;
  for (int k = lane; k < NACC * SLOT; k += 32) acc_g[k] = 0.f;
  __syncwarp();

  // CH vectors per lane are in flight at a time; with CACHE the whole row (CH == NV).
  constexpr int CH = CACHE ? NV : 4;
  const int row0 = blockIdx.x * rows_per_block;
  const int row1 = min(T, row0 + rows_per_block);
  for (int row = row0 + warp; row < row1; row += nwarps) {
    const float mean = RMS ? 0.f : mean_in[row];
    const float rstd = rstd_in[row];
    const __nv_bfloat16* xr = x + (long)row * d;
    const __nv_bfloat16* dyr = dy + (long)row * d;
    uint4 xq[CH], gq[CH];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i0 = 0; i0 < NV; i0 += CH) {
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const int c = lane + (i0 + k) * 32;
        if (c < nvec) {
          xq[k] = *reinterpret_cast<const uint4*>(xr + c * 8);
          gq[k] = *reinterpret_cast<const uint4*>(dyr + c * 8);
        }
      }
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const int i = i0 + k, c = lane + i * 32;
        if (c < nvec) {
          float xv[8], gy[8], g[8];
          unpack8(xq[k], xv);
          unpack8(gq[k], gy);
          load8(gamma + c * 8, g);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float xh = (xv[j] - mean) * rstd;
            const float w = gy[j] * g[j];
            s1 += w;
            s2 += w * xh;
            acc_g[(i * 8 + j) * 32 + lane] += gy[j] * xh;
            if (!RMS) acc_b[(i * 8 + j) * 32 + lane] += gy[j];
          }
        }
      }
    }
    const float m1 = RMS ? 0.f : warp_sum(s1) / d;
    const float m2 = warp_sum(s2) / d;
    __nv_bfloat16* dxr = dx + (long)row * d;
#pragma unroll
    for (int i0 = 0; i0 < NV; i0 += CH) {
      uint4 rq[CH];
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const int c = lane + (i0 + k) * 32;
        if (c < nvec) {
          if (!CACHE) {
            xq[k] = *reinterpret_cast<const uint4*>(xr + c * 8);
            gq[k] = *reinterpret_cast<const uint4*>(dyr + c * 8);
          }
          if (dres) rq[k] = *reinterpret_cast<const uint4*>(dres + (long)row * d + c * 8);
        }
      }
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const int c = lane + (i0 + k) * 32;
        if (c < nvec) {
          float xv[8], gy[8], g[8], o[8];
          unpack8(xq[k], xv);
          unpack8(gq[k], gy);
          load8(gamma + c * 8, g);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float xh = (xv[j] - mean) * rstd;
            o[j] = rstd * (gy[j] * g[j] - m1 - xh * m2);
          }
          if (dres) {
            float r[8];
            unpack8(rq[k], r);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] += r[j];
          }
          store8(dxr + c * 8, o);
        }
      }
    }
  }
  __syncthreads();
  for (int col = threadIdx.x; col < d; col += blockDim.x) {
    const int c = col >> 3, j = col & 7;
    const int k = ((c >> 5) * 8 + j) * 32 + (c & 31);
    float g = 0.f, b = 0.f;
    for (int w = 0; w < nwarps; ++w) {
      g += red[w * NACC * SLOT + k];
      if (!RMS) b += red[w * NACC * SLOT + SLOT + k];
    }
    atomicAdd(dgamma + col, g);
    if (!RMS && dbeta) atomicAdd(dbeta + col, b);
  }
}

template <bool RMS, int NV, bool CACHE>
int bwd_nv(const void* dy, const void* x, const void* gamma, const float* mean, const float* rstd, const void* dres,
           void* dx, float* dgamma, float* dbeta, int T, int d, cudaStream_t s) {
  constexpr int NACC = RMS ? 1 : 2;
  const size_t per_warp = (size_t)NACC * NV * 8 * 32 * sizeof(float);
  const int warps = (int)std::min<size_t>(kWarps, (200u * 1024u) / per_warp);
  const size_t smem = warps * per_warp;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int per_sm = std::max(1, (int)((220u * 1024u) / smem));
  const int blocks_target = std::min(2, per_sm) * sms;
  int rows_per_block = (T + blocks_target - 1) / blocks_target;
  rows_per_block = std::max(warps, (rows_per_block + warps - 1) / warps * warps);
  auto kern = norm_bwd_kernel<RMS, NV, CACHE>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<(T + rows_per_block - 1) / rows_per_block, warps * 32, smem, s>>>(
      (const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, (const __nv_bfloat16*)gamma, mean, rstd,
      (const __nv_bfloat16*)dres, (__nv_bfloat16*)dx, dgamma, dbeta, T, d, rows_per_block);
  return (int)cudaGetLastError();
}

template <bool RMS, int NV>
int fwd_nv(const void* x, const void* gamma, const void* beta, void* y, float* mean, float* rstd, int T, int d,
           float eps, cudaStream_t s) {
  norm_fwd_kernel<RMS, NV><<<(T + kWarps - 1) / kWarps, kWarps * 32, 0, s>>>(
      (const __nv_bfloat16*)x, (const __nv_bfloat16*)gamma, (const __nv_bfloat16*)beta, (__nv_bfloat16*)y, mean,
      rstd, T, d, eps);
  return (int)cudaGetLastError();
}

template <bool RMS>
int launch_fwd(const void* x, const void* gamma, const void* beta, void* y, float* mean, float* rstd, int T, int d,
               float eps, cudaStream_t s) {
  if (d % 8 || d > kMaxVec * 256) return -1;
  if (T == 0) return 0;
  const int nv = (d / 8 + 31) / 32;
  if (nv <= 1) return fwd_nv<RMS, 1>(x, gamma, beta, y, mean, rstd, T, d, eps, s);
  if (nv <= 2) return fwd_nv<RMS, 2>(x, gamma, beta, y, mean, rstd, T, d, eps, s);
  if (nv <= 4) return fwd_nv<RMS, 4>(x, gamma, beta, y, mean, rstd, T, d, eps, s);
  if (nv <= 6) return fwd_nv<RMS, 6>(x, gamma, beta, y, mean, rstd, T, d, eps, s);
  if (nv <= 8) return fwd_nv<RMS, 8>(x, gamma, beta, y, mean, rstd, T, d, eps, s);
  return fwd_nv<RMS, 16>(x, gamma, beta, y, mean, rstd, T, d, eps, s);
}

template <bool RMS>
int launch_bwd(const void* dy, const void* x, const void* gamma, const float* mean, const float* rstd,
               const void* dres, void* dx, float* dgamma, float* dbeta, int T, int d, cudaStream_t s) {
  if (d % 8 || d > 4096) return -1;
  if (T == 0) return 0;
  const int nv = (d / 8 + 31) / 32;
#define MT_BWD(N, C) return bwd_nv<RMS, N, C>(dy, x, gamma, mean, rstd, dres, dx, dgamma, dbeta, T, d, s)
  if (nv <= 1) MT_BWD(1, true);
  if (nv <= 2) MT_BWD(2, true);
  if (nv <= 3) MT_BWD(3, true);
  if (nv <= 4) MT_BWD(4, true);
  if (nv <= 5) MT_BWD(5, true);
  if (nv <= 6) MT_BWD(6, true);
  if (nv <= 8) MT_BWD(8, true);
  if (nv <= 12) MT_BWD(12, false);
  MT_BWD(16, false);
#undef MT_BWD
}

}  // namespace

int layernorm_fwd(const void* x, const void* gamma, const void* beta, void* y, float* mean, float* rstd, int T, int d,
                  float eps, cudaStream_t s) {
  return launch_fwd<false>(x, gamma, beta, y, mean, rstd, T, d, eps, s);
}
int layernorm_bwd(const void* dy, const void* x, const void* gamma, const float* mean, const float* rstd,
                  const void* dres, void* dx, float* dgamma, float* dbeta, int T, int d, cudaStream_t s) {
  return launch_bwd<false>(dy, x, gamma, mean, rstd, dres, dx, dgamma, dbeta, T, d, s);
}
int rmsnorm_fwd(const void* x, const void* gamma, void* y, float* rstd, int T, int d, float eps, cudaStream_t s) {
  return launch_fwd<true>(x, gamma, nullptr, y, nullptr, rstd, T, d, eps, s);
}
int rmsnorm_bwd(const void* dy, const void* x, const void* gamma, const float* rstd, const void* dres, void* dx,
                float* dgamma, int T, int d, cudaStream_t s) {
  return launch_bwd<true>(dy, x, gamma, nullptr, rstd, dres, dx, dgamma, nullptr, T, d, s);
}

}  // namespace mt
