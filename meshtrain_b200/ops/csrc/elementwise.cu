// elementwise.cu -- memory-bound fused ops: embedding gather(+pos) and its
// scatter-add backward, bias-gradient column sums, SwiGLU backward, rotary
// position embedding and fp32->bf16 casts.  All loads/stores are 16-byte vectors.
//
// Replaces nn.Embedding + positional add (reference models/tiny_transformer.py:19-27)
// and the ATen reductions autograd runs for Linear bias gradients.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include <mutex>

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
  MT_CHECK(id >= 0 && id < V, kErrCheckIndex);  // debug builds record an out-of-range token id
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
  MT_CHECK(id >= 0 && id < V, kErrCheckIndex);
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

// ---------------------------------------------------------------------------
// Deterministic embedding backward: the same gradient rows summed in the same
// order on every run, with no atomics.
//
//  1. embed_sort_kernel (one CTA): keys (id << 15 | t) sorted by a bitonic
//     sort in shared memory, so positions with equal ids end up adjacent and in
//     increasing t; it writes the sorted positions, the start of every run of
//     equal ids (a block-wide scan of the run-start flags) and the run count.
//  2. embed_runs_kernel: one warp per run sums dy[t] of its positions in t order
//     and adds the sum to tok_grad[id]: every row has exactly one writer.
//  3. embed_pos_kernel: one warp per position p sums dy[b*S + p] over the
//     sequences b in order into pos_grad[p].
// Keys are 32-bit: T <= 32768 positions and V <= 131072 rows.
constexpr int kSortThreads = 1024;
constexpr int kSortMaxT = 32768;
constexpr int kSortTBits = 15;

__global__ void __launch_bounds__(kSortThreads) embed_sort_kernel(const int64_t* __restrict__ ids, int T, int V, int N,
                                                                 int* __restrict__ sorted_t, int* __restrict__ runs,
                                                                 int* __restrict__ nruns) {
  extern __shared__ uint32_t keys[];  // N (power of two) keys, then kSortThreads scan slots
  uint32_t* scan = keys + N;
  const int tid = threadIdx.x;
  for (int i = tid; i < N; i += kSortThreads) {
    if (i < T) {
      long id = ids[i];
      MT_CHECK(id >= 0 && id < V, kErrCheckIndex);
      id = id < 0 ? 0 : (id >= V ? V - 1 : id);
      keys[i] = ((uint32_t)id << kSortTBits) | (uint32_t)i;
    } else {
      keys[i] = 0xFFFFFFFFu;  // padding sorts last
    }
  }
  __syncthreads();
  for (int size = 2; size <= N; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < N / 2; i += kSortThreads) {
        // the i-th compare-exchange pair of this pass
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool ascending = (lo & size) == 0;
        const uint32_t a = keys[lo], b = keys[hi];
        if ((a > b) == ascending) {
          keys[lo] = b;
          keys[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  // run starts: i == 0 or a new id; each thread counts a contiguous slice, then a block scan
  const int per = (T + kSortThreads - 1) / kSortThreads;
  const int b0 = min(T, tid * per), b1 = min(T, b0 + per);
  uint32_t count = 0;
  for (int i = b0; i < b1; ++i) count += (i == 0 || (keys[i] >> kSortTBits) != (keys[i - 1] >> kSortTBits)) ? 1u : 0u;
  scan[tid] = count;
  __syncthreads();
  for (int off = 1; off < kSortThreads; off <<= 1) {  // inclusive Hillis-Steele scan
    const uint32_t v = tid >= off ? scan[tid - off] : 0u;
    __syncthreads();
    scan[tid] += v;
    __syncthreads();
  }
  uint32_t pos = scan[tid] - count;
  for (int i = b0; i < b1; ++i) {
    sorted_t[i] = (int)(keys[i] & ((1u << kSortTBits) - 1));
    if (i == 0 || (keys[i] >> kSortTBits) != (keys[i - 1] >> kSortTBits)) runs[pos++] = i;
  }
  if (tid == kSortThreads - 1) {
    *nruns = (int)scan[kSortThreads - 1];
    runs[scan[kSortThreads - 1]] = T;  // sentinel end of the last run
  }
}

__global__ void embed_runs_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ dy,
                                  const int* __restrict__ sorted_t, const int* __restrict__ runs,
                                  const int* __restrict__ nruns, float* __restrict__ tok_grad, int d, int V) {
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= *nruns) return;
  const int s = runs[r], e = runs[r + 1];
  long id = ids[sorted_t[s]];
  id = id < 0 ? 0 : (id >= V ? V - 1 : id);
  float* row = tok_grad + id * (long)d;
  for (int c = lane * 8; c < d; c += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int i = s; i < e; ++i) {
      float a[8];
      ld8(dy + (long)sorted_t[i] * d + c, a);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += a[j];
    }
    float4* out = reinterpret_cast<float4*>(row + c);
    float4 lo = out[0], hi = out[1];
    out[0] = make_float4(lo.x + acc[0], lo.y + acc[1], lo.z + acc[2], lo.w + acc[3]);
    out[1] = make_float4(hi.x + acc[4], hi.y + acc[5], hi.z + acc[6], hi.w + acc[7]);
  }
}

__global__ void embed_pos_kernel(const __nv_bfloat16* __restrict__ dy, float* __restrict__ pos_grad, int T, int S,
                                 int d) {
  const int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (p >= S) return;
  for (int c = lane * 8; c < d; c += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int t = p; t < T; t += S) {
      float a[8];
      ld8(dy + (long)t * d + c, a);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += a[j];
    }
    float4* out = reinterpret_cast<float4*>(pos_grad + (long)p * d + c);
    float4 lo = out[0], hi = out[1];
    out[0] = make_float4(lo.x + acc[0], lo.y + acc[1], lo.z + acc[2], lo.w + acc[3]);
    out[1] = make_float4(hi.x + acc[4], hi.y + acc[5], hi.z + acc[6], hi.w + acc[7]);
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

int embedding_bwd_sorted_scratch_ints(int T) { return 2 * T + 2; }

int embedding_bwd_sorted(const int64_t* ids, const void* dy, float* tok_grad, float* pos_grad, int T, int S, int d,
                         int V, int* scratch, cudaStream_t s) {
  if (d % 8 || T > kSortMaxT || V > (1 << (32 - kSortTBits))) return -1;
  if (T == 0) return 0;
  int N = 1;
  while (N < T) N <<= 1;
  const int smem = (N + kSortThreads) * (int)sizeof(uint32_t);
  static std::once_flag attr_flags[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(attr_flags[dev & 63], [] {
    cudaFuncSetAttribute(embed_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (kSortMaxT + kSortThreads) * (int)sizeof(uint32_t));
  });
  int* sorted_t = scratch;
  int* runs = scratch + T;          // T + 1 entries (run starts + end sentinel)
  int* nruns = scratch + 2 * T + 1;
  embed_sort_kernel<<<1, kSortThreads, smem, s>>>(ids, T, V, N, sorted_t, runs, nruns);
  embed_runs_kernel<<<(T + 7) / 8, 256, 0, s>>>(ids, (const __nv_bfloat16*)dy, sorted_t, runs, nruns, tok_grad, d, V);
  if (pos_grad != nullptr && S > 0) embed_pos_kernel<<<(S + 7) / 8, 256, 0, s>>>((const __nv_bfloat16*)dy, pos_grad, T, S, d);
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
