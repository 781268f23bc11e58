// adam.cu -- fused multi-tensor Adam / AdamW over one flat parameter buffer.
//
// A stage keeps all of its parameters in one contiguous fp32 master buffer (and
// its gradients, exp_avg and exp_avg_sq in buffers of the same layout), so one
// launch updates everything: read p, g, m, v; write p, m, v and the bf16
// compute copy.  Semantics follow torch.optim.Adam/AdamW (reference
// runtime/stage.py:28-36): L2 decay folded into g for Adam, decoupled decay for
// AdamW, bias corrections precomputed on the host.
#include <cuda_bf16.h>
#include <algorithm>
#include <cuda_runtime.h>

#include "mt_api.h"
#include "sm100.cuh"

namespace mt {
namespace {

struct AdamHyper {
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, grad_scale;
  bool decoupled;
};

__device__ __forceinline__ void adam_one(float& p, float g, float& m, float& v, const AdamHyper& h) {
  g *= h.grad_scale;
  if (h.decoupled) p *= 1.f - h.lr * h.wd;
  else g += h.wd * p;
  m = h.beta1 * m + (1.f - h.beta1) * g;
  v = h.beta2 * v + (1.f - h.beta2) * g * g;
  const float denom = sqrtf(v) / h.bc2_sqrt + h.eps;
  p -= (h.lr / h.bc1) * (m / denom);
}

__global__ void adam_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                            float* __restrict__ v, __nv_bfloat16* __restrict__ pb, long n, AdamHyper h) {
  const long stride = (long)gridDim.x * blockDim.x * 4;
  for (long i = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < n; i += stride) {
    if (i + 4 <= n) {
      float4 P = *reinterpret_cast<float4*>(p + i);
      const float4 G = *reinterpret_cast<const float4*>(g + i);
      float4 Mv = *reinterpret_cast<float4*>(m + i);
      float4 Vv = *reinterpret_cast<float4*>(v + i);
      adam_one(P.x, G.x, Mv.x, Vv.x, h);
      adam_one(P.y, G.y, Mv.y, Vv.y, h);
      adam_one(P.z, G.z, Mv.z, Vv.z, h);
      adam_one(P.w, G.w, Mv.w, Vv.w, h);
      *reinterpret_cast<float4*>(p + i) = P;
      *reinterpret_cast<float4*>(m + i) = Mv;
      *reinterpret_cast<float4*>(v + i) = Vv;
      if (pb) {
        *reinterpret_cast<uint2*>(pb + i) = make_uint2(pack_bf16x2(P.x, P.y), pack_bf16x2(P.z, P.w));
      }
    } else {
      for (long j = i; j < n; ++j) {
        float P = p[j], Mv = m[j], Vv = v[j];
        adam_one(P, g[j], Mv, Vv, h);
        p[j] = P;
        m[j] = Mv;
        v[j] = Vv;
        if (pb) pb[j] = __float2bfloat16_rn(P);
      }
    }
  }
}

}  // namespace

int adam_step(float* param, const float* grad, float* exp_avg, float* exp_avg_sq, void* param_bf16, long n, float lr,
              float beta1, float beta2, float eps, float weight_decay, bool decoupled, float bias_correction1,
              float bias_correction2, float grad_scale, cudaStream_t s) {
  if (n == 0) return 0;
  AdamHyper h{lr, beta1, beta2, eps, weight_decay, bias_correction1, sqrtf(bias_correction2), grad_scale, decoupled};
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long vec = (n + 3) / 4;
  const long blocks = std::min<long>((vec + 255) / 256, (long)sms * 8);
  adam_kernel<<<(unsigned)blocks, 256, 0, s>>>(param, grad, exp_avg, exp_avg_sq, (__nv_bfloat16*)param_bf16, n, h);
  return (int)cudaGetLastError();
}

}  // namespace mt
