// cross_entropy.cu -- fused softmax cross-entropy forward + backward over a
// chunk of bf16 logits, in place.
//
// One block per token row: pass 1 keeps a per-thread online (max, sum-exp),
// reduces them across the block and forms logsumexp; pass 2 overwrites the row
// with dlogits = (softmax - onehot) * grad_scale.  The caller feeds it one
// token chunk of LM-head logits at a time, so the full [tokens, vocab] fp32
// logits the reference materialises (models/tiny_transformer.py:93-94,
// F.cross_entropy(output.float())) never exist.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "mt_api.h"
#include "sm100.cuh"

namespace mt {
namespace {

constexpr int kThreads = 512;

__device__ __forceinline__ void merge(float& m, float& s, float m2, float s2) {
  if (m2 > m) {
    s = s * __expf(m - m2) + s2;
    m = m2;
  } else if (m2 > -INFINITY) {
    s += s2 * __expf(m2 - m);
  }
}

__global__ void __launch_bounds__(kThreads) ce_kernel(__nv_bfloat16* __restrict__ logits, long ld,
                                                      const int64_t* __restrict__ targets, float* __restrict__ loss_sum,
                                                      int V, float loss_scale, float grad_scale) {
  __shared__ float sm_m[kThreads / 32], sm_s[kThreads / 32];
  __shared__ float sh_lse;
  const long row = blockIdx.x;
  __nv_bfloat16* x = logits + row * ld;
  const int64_t tgt = targets[row];
  if (threadIdx.x == 0) MT_CHECK(tgt >= 0 && tgt < V, kErrCheckIndex);  // such rows add no loss or gradient
  const int nvec = V / 8;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x; c < nvec; c += kThreads) {
    uint4 q = *reinterpret_cast<const uint4*>(x + c * 8);
    uint32_t w[4] = {q.x, q.y, q.z, q.w};
    float f[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 t = unpack_bf16x2(w[j]);
      f[2 * j] = t.x;
      f[2 * j + 1] = t.y;
    }
    float lm = f[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) lm = fmaxf(lm, f[j]);
    float ls = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ls += __expf(f[j] - lm);
    merge(m, s, lm, ls);
  }
  for (int c = nvec * 8 + threadIdx.x; c < V; c += kThreads) merge(m, s, __bfloat162float(x[c]), 1.f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge(m, s, m2, s2);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm_m[warp] = m;
    sm_s[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm_m[0], Ssum = sm_s[0];
    for (int w = 1; w < kThreads / 32; ++w) merge(M, Ssum, sm_m[w], sm_s[w]);
    const float lse = M + logf(Ssum);
    sh_lse = lse;
    if (tgt >= 0 && tgt < V) atomicAdd(loss_sum, (lse - __bfloat162float(x[tgt])) * loss_scale);
  }
  __syncthreads();
  const float lse = sh_lse;
  const bool valid = tgt >= 0 && tgt < V;
  const float gs = valid ? grad_scale : 0.f;
  for (int c = threadIdx.x; c < nvec; c += kThreads) {
    uint4 q = *reinterpret_cast<const uint4*>(x + c * 8);
    uint32_t w[4] = {q.x, q.y, q.z, q.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 t = unpack_bf16x2(w[j]);
      const int col = c * 8 + 2 * j;
      float g0 = __expf(t.x - lse) - (col == tgt ? 1.f : 0.f);
      float g1 = __expf(t.y - lse) - (col + 1 == tgt ? 1.f : 0.f);
      o[j] = pack_bf16x2(g0 * gs, g1 * gs);
    }
    *reinterpret_cast<uint4*>(x + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  for (int c = nvec * 8 + threadIdx.x; c < V; c += kThreads) {
    const float t = __bfloat162float(x[c]);
    x[c] = __float2bfloat16_rn((__expf(t - lse) - (c == tgt ? 1.f : 0.f)) * gs);
  }
}

}  // namespace

int cross_entropy_fwd_bwd(void* logits, long ld, const int64_t* targets, float* loss_sum, int T, int V,
                          float loss_scale, float grad_scale, cudaStream_t s) {
  if (ld % 8) return -1;
  if (T == 0) return 0;
  ce_kernel<<<T, kThreads, 0, s>>>((__nv_bfloat16*)logits, ld, targets, loss_sum, V, loss_scale, grad_scale);
  return (int)cudaGetLastError();
}

}  // namespace mt
