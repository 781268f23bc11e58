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

// Backward: two passes over each row (the second hits L1), parameter-gradient
// partials accumulated per warp in shared memory, then one atomic per column
// per block into the fp32 accumulators.
template <bool RMS>
__global__ void __launch_bounds__(kWarps * 32)
    norm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                    const __nv_bfloat16* __restrict__ gamma, const float* __restrict__ mean_in,
                    const float* __restrict__ rstd_in, const __nv_bfloat16* __restrict__ dres,
                    __nv_bfloat16* __restrict__ dx, float* __restrict__ dgamma, float* __restrict__ dbeta,
                    int T, int d, int rows_per_block) {
  extern __shared__ float red[];  // [warps][2][d]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int nvec = d >> 3;
  float* rg = red + warp * 2 * d;
  float* rb = rg + d;
  for (int c = lane; c < d; c += 32) rg[c] = rb[c] = 0.f;
  __syncwarp();

  const int row0 = blockIdx.x * rows_per_block;
  const int row1 = min(T, row0 + rows_per_block);
  for (int row = row0 + warp; row < row1; row += nwarps) {
    const float mean = RMS ? 0.f : mean_in[row];
    const float rstd = rstd_in[row];
    const __nv_bfloat16* xr = x + (long)row * d;
    const __nv_bfloat16* dyr = dy + (long)row * d;
    float s1 = 0.f, s2 = 0.f;
    for (int c = lane; c < nvec; c += 32) {
      float xv[8], g[8], gy[8];
      load8(xr + c * 8, xv);
      load8(dyr + c * 8, gy);
      load8(gamma + c * 8, g);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = (xv[j] - mean) * rstd;
        const float w = gy[j] * g[j];
        s1 += w;
        s2 += w * xh;
        rg[c * 8 + j] += gy[j] * xh;
        rb[c * 8 + j] += gy[j];
      }
    }
    const float m1 = RMS ? 0.f : warp_sum(s1) / d;
    const float m2 = warp_sum(s2) / d;
    __nv_bfloat16* dxr = dx + (long)row * d;
    for (int c = lane; c < nvec; c += 32) {
      float xv[8], g[8], gy[8], o[8], r[8];
      load8(xr + c * 8, xv);
      load8(dyr + c * 8, gy);
      load8(gamma + c * 8, g);
      if (dres) load8(dres + (long)row * d + c * 8, r);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = (xv[j] - mean) * rstd;
        o[j] = rstd * (gy[j] * g[j] - m1 - xh * m2);
        if (dres) o[j] += r[j];
      }
      store8(dxr + c * 8, o);
    }
  }
  __syncthreads();
  for (int col = threadIdx.x; col < d; col += blockDim.x) {
    float g = 0.f, b = 0.f;
    for (int w = 0; w < nwarps; ++w) {
      g += red[w * 2 * d + col];
      b += red[w * 2 * d + d + col];
    }
    atomicAdd(dgamma + col, g);
    if (!RMS && dbeta) atomicAdd(dbeta + col, b);
  }
}

// Backward for rows of up to 6 x 256 elements: each lane owns the same
// columns of every row it visits, so dgamma/dbeta partials stay in registers
// across rows; one cross-warp reduction and one atomic per column per block.
template <bool RMS, int NV>
__global__ void __launch_bounds__(kWarps * 32)
    norm_bwd_reg_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                        const __nv_bfloat16* __restrict__ gamma, const float* __restrict__ mean_in,
                        const float* __restrict__ rstd_in, const __nv_bfloat16* __restrict__ dres,
                        __nv_bfloat16* __restrict__ dx, float* __restrict__ dgamma, float* __restrict__ dbeta,
                        int T, int d, int rows_per_block) {
  extern __shared__ float red[];  // [2][d]: block partial dgamma, dbeta
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = d >> 3;
  for (int c = threadIdx.x; c < 2 * d; c += blockDim.x) red[c] = 0.f;
  __syncthreads();
  float pg[NV][8], pb[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) pg[i][j] = pb[i][j] = 0.f;
  const int row0 = blockIdx.x * rows_per_block;
  const int row1 = min(T, row0 + rows_per_block);
  for (int row = row0 + warp; row < row1; row += kWarps) {
    const float mean = RMS ? 0.f : mean_in[row];
    const float rstd = rstd_in[row];
    const __nv_bfloat16* xr = x + (long)row * d;
    const __nv_bfloat16* dyr = dy + (long)row * d;
    float xh[NV][8], gy[NV][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = lane + i * 32;
      if (c < nvec) {
        float g[8];
        load8(xr + c * 8, xh[i]);
        load8(dyr + c * 8, gy[i]);
        load8(gamma + c * 8, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[i][j] = (xh[i][j] - mean) * rstd;
          const float w = gy[i][j] * g[j];
          s1 += w;
          s2 += w * xh[i][j];
          pg[i][j] += gy[i][j] * xh[i][j];
          pb[i][j] += gy[i][j];
        }
      }
    }
    const float m1 = RMS ? 0.f : warp_sum(s1) / d;
    const float m2 = warp_sum(s2) / d;
    __nv_bfloat16* dxr = dx + (long)row * d;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = lane + i * 32;
      if (c < nvec) {
        float g[8], o[8], r[8];
        load8(gamma + c * 8, g);
        if (dres) load8(dres + (long)row * d + c * 8, r);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j] = rstd * (gy[i][j] * g[j] - m1 - xh[i][j] * m2);
          if (dres) o[j] += r[j];
        }
        store8(dxr + c * 8, o);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        atomicAdd(&red[c * 8 + j], pg[i][j]);
        if (!RMS) atomicAdd(&red[d + c * 8 + j], pb[i][j]);
      }
    }
  }
  __syncthreads();
  for (int col = threadIdx.x; col < d; col += blockDim.x) {
    atomicAdd(dgamma + col, red[col]);
    if (!RMS && dbeta) atomicAdd(dbeta + col, red[d + col]);
  }
}

template <bool RMS, int NV>
int bwd_reg(const void* dy, const void* x, const void* gamma, const float* mean, const float* rstd, const void* dres,
            void* dx, float* dgamma, float* dbeta, int T, int d, cudaStream_t s) {
  // ~4 blocks per SM: enough rows per block to amortise the parameter-gradient
  // atomics, enough blocks to fill the GPU.
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int rows_per_block = (T + 4 * sms - 1) / (4 * sms);
  rows_per_block = std::max(kWarps, (rows_per_block + kWarps - 1) / kWarps * kWarps);
  const size_t smem = (size_t)2 * d * sizeof(float);
  auto kern = norm_bwd_reg_kernel<RMS, NV>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<(T + rows_per_block - 1) / rows_per_block, kWarps * 32, smem, s>>>(
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
  if (d % 8 || d > 6144) return -1;
  if (T == 0) return 0;
  const int nv = (d / 8 + 31) / 32;
  if (nv <= 2) return bwd_reg<RMS, 2>(dy, x, gamma, mean, rstd, dres, dx, dgamma, dbeta, T, d, s);
  if (nv <= 4) return bwd_reg<RMS, 4>(dy, x, gamma, mean, rstd, dres, dx, dgamma, dbeta, T, d, s);
  if (nv <= 6) return bwd_reg<RMS, 6>(dy, x, gamma, mean, rstd, dres, dx, dgamma, dbeta, T, d, s);
  const int rows_per_block = 128;
  const int warps = d > 2048 ? 4 : kWarps;  // keep the partial sums under 227 KB of shared memory
  const size_t smem = (size_t)warps * 2 * d * sizeof(float);
  auto kern = norm_bwd_kernel<RMS>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<(T + rows_per_block - 1) / rows_per_block, warps * 32, smem, s>>>(
      (const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, (const __nv_bfloat16*)gamma, mean, rstd,
      (const __nv_bfloat16*)dres, (__nv_bfloat16*)dx, dgamma, dbeta, T, d, rows_per_block);
  return (int)cudaGetLastError();
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
