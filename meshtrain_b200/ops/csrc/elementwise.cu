// elementwise.cu -- memory-bound fused ops: embedding gather(+pos) and its
// scatter-add backward, bias-gradient column sums, SwiGLU backward, rotary
// position embedding and fp32->bf16 casts.  All loads/stores are 16-byte vectors.
//
// Replaces nn.Embedding + positional add (reference models/tiny_transformer.py:19-27)
// and the ATen reductions autograd runs for Linear bias gradients.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "mt_api.h"
#include "sm100.cuh"

namespace mt {
namespace {

__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float* f) {
  uint4 q = *reinterpret_cast<const uint4*>(p);
  uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 t = unpack_bf16x2(w[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}
__device__ __forceinline__ void st8(__nv_bfloat16* p, const float* f) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                            pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
}

// one warp per token
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ tok,
                                     const __nv_bfloat16* __restrict__ pos, __nv_bfloat16* __restrict__ out, int T,
                                     int S, int d, int V) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  long id = ids[t];
  id = id < 0 ? 0 : (id >= V ? V - 1 : id);  // the launcher validates ids; clamp keeps reads in bounds
  const __nv_bfloat16* tr = tok + id * (long)d;
  const __nv_bfloat16* pr = pos ? pos + (long)(t % S) * d : nullptr;
  __nv_bfloat16* o = out + (long)t * d;
  for (int c = lane * 8; c < d; c += 256) {
    float a[8];
    ld8(tr + c, a);
    if (pr) {
      float b[8];
      ld8(pr + c, b);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] += b[j];
    }
    st8(o + c, a);
  }
}

__device__ __forceinline__ void atomic_add4(float* p, float a, float b, float c, float d) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
  atomicAdd(reinterpret_cast<float4*>(p), make_float4(a, b, c, d));
#else
  atomicAdd(p, a); atomicAdd(p + 1, b); atomicAdd(p + 2, c); atomicAdd(p + 3, d);
#endif
}

__global__ void embedding_bwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ dy,
                                     float* __restrict__ tok_grad, float* __restrict__ pos_grad, int T, int S, int d,
                                     int V) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  long id = ids[t];
  id = id < 0 ? 0 : (id >= V ? V - 1 : id);
  const __nv_bfloat16* g = dy + (long)t * d;
  float* tg = tok_grad + id * (long)d;
  float* pg = pos_grad ? pos_grad + (long)(t % S) * d : nullptr;
  for (int c = lane * 8; c < d; c += 256) {
    float a[8];
    ld8(g + c, a);
    atomic_add4(tg + c, a[0], a[1], a[2], a[3]);
    atomic_add4(tg + c + 4, a[4], a[5], a[6], a[7]);
    if (pg) {
      atomic_add4(pg + c, a[0], a[1], a[2], a[3]);
      atomic_add4(pg + c + 4, a[4], a[5], a[6], a[7]);
    }
  }
}

// out[n] += sum_t dy[t,n] (bias gradients).  A block is 32 column threads x 8
// row groups: a column thread owns 8 adjacent columns (one 16-byte load per
// row), so a warp reads 512 contiguous bytes of a row and a block covers 256
// columns.  Each thread keeps 4 row loads in flight; the 8 row groups are
// summed in shared memory and the block adds one value per column.
constexpr int kCsCols = 32, kCsGroups = 8, kCsUnroll = 4;

__global__ void __launch_bounds__(kCsCols * kCsGroups)
    colsum_kernel(const __nv_bfloat16* __restrict__ dy, long ld, float* __restrict__ out, int T, int N,
                  int rows_per_block) {
  __shared__ float part[kCsGroups][kCsCols * 8];
  const int ct = threadIdx.x % kCsCols, rg = threadIdx.x / kCsCols;
  const int col = (blockIdx.x * kCsCols + ct) * 8;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(T, r0 + rows_per_block);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (col + 8 <= N) {
    int r = r0 + rg;
    for (; r + (kCsUnroll - 1) * kCsGroups < r1; r += kCsUnroll * kCsGroups) {
      uint4 q[kCsUnroll];
#pragma unroll
      for (int u = 0; u < kCsUnroll; ++u)
        q[u] = *reinterpret_cast<const uint4*>(dy + (long)(r + u * kCsGroups) * ld + col);
#pragma unroll
      for (int u = 0; u < kCsUnroll; ++u) {
        const uint32_t w[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack_bf16x2(w[k]);
          acc[2 * k] += f.x;
          acc[2 * k + 1] += f.y;
        }
      }
    }
    for (; r < r1; r += kCsGroups) {
      float f[8];
      ld8(dy + (long)r * ld + col, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += f[j];
    }
  } else {
    for (int r = r0 + rg; r < r1; r += kCsGroups)
      for (int j = 0; j < 8 && col + j < N; ++j) acc[j] += __bfloat162float(dy[(long)r * ld + col + j]);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) part[rg][ct * 8 + j] = acc[j];
  __syncthreads();
  const int c = threadIdx.x;  // 256 threads, 256 columns
  const int gcol = blockIdx.x * kCsCols * 8 + c;
  if (gcol < N) {
    float sum = 0.f;
#pragma unroll
    for (int g = 0; g < kCsGroups; ++g) sum += part[g][c];
    atomicAdd(out + gcol, sum);
  }
}

// raw/draw: [T, 2F] with blocks of 32 columns = [16 gate | 16 up] for 16 features.
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ raw,
                                  __nv_bfloat16* __restrict__ draw, int T, int F) {
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;  // one thread per 8 features
  const long per_row = F / 8;
  if (idx >= (long)T * per_row) return;
  const long t = idx / per_row;
  const int f0 = (int)(idx - t * per_row) * 8;
  const int blk = f0 / 16, i0 = f0 % 16;
  const long gofs = t * 2L * F + blk * 32 + i0;
  float g[8], u[8], d[8], dg[8], du[8];
  ld8(raw + gofs, g);
  ld8(raw + gofs + 16, u);
  ld8(dout + t * (long)F + f0, d);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float sg = 1.0f / (1.0f + __expf(-g[j]));
    const float s = g[j] * sg;
    du[j] = d[j] * s;
    dg[j] = d[j] * u[j] * (sg * (1.0f + g[j] * (1.0f - sg)));
  }
  st8(draw + gofs, dg);
  st8(draw + gofs + 16, du);
}

// Rotate-half RoPE on the first H heads of each packed row (in place).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ qk, long ld, int T, int S, int H, int hd, float theta,
                            float sign) {
  const int half = hd / 2;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)T * H * half) return;
  const int i = (int)(idx % half);
  const long th = idx / half;
  const int h = (int)(th % H);
  const long t = th / H;
  const int pos = (int)(t % S);
  const float inv_freq = powf(theta, -2.0f * (float)i / (float)hd);
  float sn, cs;
  sincosf((float)pos * inv_freq, &sn, &cs);
  sn *= sign;
  __nv_bfloat16* p = qk + t * ld + (long)h * hd;
  const float x1 = __bfloat162float(p[i]);
  const float x2 = __bfloat162float(p[i + half]);
  p[i] = __float2bfloat16_rn(x1 * cs - x2 * sn);
  p[i + half] = __float2bfloat16_rn(x2 * cs + x1 * sn);
}

__global__ void cast_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out, long n) {
  const long i = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i + 8 <= n) {
    float4 a = *reinterpret_cast<const float4*>(in + i);
    float4 b = *reinterpret_cast<const float4*>(in + i + 4);
    float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    st8(out + i, f);
  } else {
    for (long j = i; j < n; ++j) out[j] = __float2bfloat16_rn(in[j]);
  }
}

}  // namespace

int embedding_fwd(const int64_t* ids, const void* tok, const void* pos, void* out, int T, int S, int d, int V,
                  cudaStream_t s) {
  if (d % 8) return -1;
  if (T == 0) return 0;
  embedding_fwd_kernel<<<(T + 7) / 8, 256, 0, s>>>(ids, (const __nv_bfloat16*)tok, (const __nv_bfloat16*)pos,
                                                   (__nv_bfloat16*)out, T, S, d, V);
  return (int)cudaGetLastError();
}

int embedding_bwd(const int64_t* ids, const void* dy, float* tok_grad, float* pos_grad, int T, int S, int d, int V,
                  cudaStream_t s) {
  if (d % 8) return -1;
  if (T == 0) return 0;
  embedding_bwd_kernel<<<(T + 7) / 8, 256, 0, s>>>(ids, (const __nv_bfloat16*)dy, tok_grad, pos_grad, T, S, d, V);
  return (int)cudaGetLastError();
}

int colsum_accumulate(const void* dy, long ld, float* out, int T, int N, cudaStream_t s) {
  if (T == 0 || N == 0) return 0;
  if (ld % 8) return -1;  // 16-byte row alignment (every caller's buffers are padded to it)
  const int col_blocks = (N + kCsCols * 8 - 1) / (kCsCols * 8);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // about 4 blocks per SM in total, at least 64 rows per block
  const int row_blocks = std::max(1, std::min((T + 63) / 64, (4 * sms + col_blocks - 1) / col_blocks));
  const int rows = (T + row_blocks - 1) / row_blocks;
  dim3 grid(col_blocks, (T + rows - 1) / rows);
  colsum_kernel<<<grid, kCsCols * kCsGroups, 0, s>>>((const __nv_bfloat16*)dy, ld, out, T, N, rows);
  return (int)cudaGetLastError();
}

int swiglu_bwd(const void* dout, const void* raw, void* draw, int T, int F, cudaStream_t s) {
  if (F % 16) return -1;
  const long n = (long)T * (F / 8);
  if (n == 0) return 0;
  swiglu_bwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((const __nv_bfloat16*)dout,
                                                                (const __nv_bfloat16*)raw, (__nv_bfloat16*)draw, T, F);
  return (int)cudaGetLastError();
}

int rope_apply(void* qk, long ld, int T, int S, int H, int hd, float theta, bool inverse, cudaStream_t s) {
  if (hd % 2) return -1;
  const long n = (long)T * H * (hd / 2);
  if (n == 0) return 0;
  rope_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((__nv_bfloat16*)qk, ld, T, S, H, hd, theta,
                                                          inverse ? -1.f : 1.f);
  return (int)cudaGetLastError();
}

int cast_f32_bf16(const float* in, void* out, long n, cudaStream_t s) {
  if (n == 0) return 0;
  const long threads = (n + 7) / 8;
  cast_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(in, (__nv_bfloat16*)out, n);
  return (int)cudaGetLastError();
}

}  // namespace mt
