// mt_api.h -- torch-free host API of the meshtrain_b200 CUDA kernels.
//
// The kernels (*.cu) include only CUDA headers so they compile quickly and can
// be linked into any host program; bindings.cpp adapts them to torch tensors.
// Every launcher returns 0 on success or a cudaError_t / negative code, and
// writes a one-line message into `err` on failure.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mt {

// ------------------------------------------------------------------ status
// One 32-bit status word per device.  A kernel that runs out of its wait
// budget ORs an error code (see sm100.cuh) into it instead of hanging.
uint32_t* device_status(int device);
uint32_t read_and_clear_status(int device);
// Debug builds (-DMT_DEBUG_CHECKS): OR of every kernel unit's failed-check codes
// (kErrCheck* in sm100.cuh), cleared by the read; always 0 in release builds.
uint32_t read_and_clear_checks();
bool debug_checks_built();

// ------------------------------------------------------------------ GEMM
struct GemmArgs {
  const void* a;  // bf16; [M,K] if !a_mn else [K,M]; leading dim lda (elements)
  long lda;
  bool a_mn;
  const void* b;  // bf16; [N,K] if !b_mn else [K,N]
  long ldb;
  bool b_mn;
  int M, N, K;
  int epi;        // mt::Epi
  void* d;        // bf16 (fp32 for kEpiF32)
  long ldd;
  void* d2;       // second bf16 output (GELU pre-activation / SwiGLU raw)
  long ldd2;
  const void* bias;  // bf16 [N] or null
  const void* aux;   // bf16 residual or saved pre-activation
  long ldaux;
  float beta;        // fp32 epilogue: D = beta * D + acc
};
int gemm_launch(const GemmArgs& args, int device, cudaStream_t stream, char* err, int errlen);

// ------------------------------------------------------------------ norms
// LayerNorm over the last dim (d) of x[T,d]; saves fp32 mean/rstd per row.
int layernorm_fwd(const void* x, const void* gamma, const void* beta, void* y, float* mean, float* rstd, int T, int d,
                  float eps, cudaStream_t s);
// dx = LN'(dy) (+ dres); dgamma/dbeta accumulate into fp32 buffers.
int layernorm_bwd(const void* dy, const void* x, const void* gamma, const float* mean, const float* rstd,
                  const void* dres, void* dx, float* dgamma, float* dbeta, int T, int d, cudaStream_t s);
int rmsnorm_fwd(const void* x, const void* gamma, void* y, float* rstd, int T, int d, float eps, cudaStream_t s);
int rmsnorm_bwd(const void* dy, const void* x, const void* gamma, const float* rstd, const void* dres, void* dx,
                float* dgamma, int T, int d, cudaStream_t s);

// ------------------------------------------------------------------ elementwise
// out[t,:] = tok[ids[t],:] (+ pos[t % S,:]); bf16.
int embedding_fwd(const int64_t* ids, const void* tok, const void* pos, void* out, int T, int S, int d, int V,
                  cudaStream_t s);
// tok_grad[ids[t],:] += dy[t,:]; pos_grad[t % S,:] += dy[t,:]  (fp32 accumulators)
// Deterministic variant (no atomics): needs T <= 32768, V <= 131072 and a scratch of
// embedding_bwd_sorted_scratch_ints(T) ints on the device.
int embedding_bwd_sorted_scratch_ints(int T);
int embedding_bwd_sorted(const int64_t* ids, const void* dy, float* tok_grad, float* pos_grad, int T, int S, int d,
                         int V, int* scratch, cudaStream_t s);
int embedding_bwd(const int64_t* ids, const void* dy, float* tok_grad, float* pos_grad, int T, int S, int d, int V,
                  cudaStream_t s);
// out[n] += sum_t dy[t, n]  (fp32 accumulator)
int colsum_accumulate(const void* dy, long ld, float* out, int T, int N, cudaStream_t s);
// SwiGLU backward on interleaved [16 gate | 16 up] blocks of raw[T, 2F].
int swiglu_bwd(const void* dout, const void* raw, void* draw, int T, int F, cudaStream_t s);
// Rotary embedding on q [T, Hq, hd] and k [T, Hk, hd] inside a packed row of width `ld`.
int rope_apply(void* qk, long ld, int T, int S, int H, int hd, float theta, bool inverse, cudaStream_t s);

// ------------------------------------------------------------------ loss
// Cross-entropy over bf16 logits [T, V] (leading dim ld), in place: logits become
// dlogits = (softmax - onehot) * grad_scale; loss_sum += sum_t ce_t * loss_scale.
int cross_entropy_fwd_bwd(void* logits, long ld, const int64_t* targets, float* loss_sum, int T, int V,
                          float loss_scale, float grad_scale, cudaStream_t s);

// ------------------------------------------------------------------ optimizer
// Fused Adam/AdamW over flat fp32 arrays; optional bf16 copy-out of the params.
int adam_step(float* param, const float* grad, float* exp_avg, float* exp_avg_sq, void* param_bf16, long n, float lr,
              float beta1, float beta2, float eps, float weight_decay, bool decoupled, float bias_correction1,
              float bias_correction2, float grad_scale, cudaStream_t s);
// out_bf16[i] = bf16(in_f32[i])
int cast_f32_bf16(const float* in, void* out, long n, cudaStream_t s);

// ------------------------------------------------------------------ attention
struct AttnArgs {
  const void* q;  // bf16 [B, S, Hq, hd] inside rows of width ld_q (elements)
  const void* k;  // bf16 [B, S, Hk, hd]
  const void* v;
  long ld_q, ld_k, ld_v;  // row stride (elements) of one token
  void* o;        // bf16 [B, S, Hq, hd], row stride ld_o
  long ld_o;
  float* lse;     // fp32 [B, Hq, S] (natural-log logsumexp of scaled scores)
  int B, S, Hq, Hk, hd;
  float scale;
  bool causal;
};
int attention_fwd(const AttnArgs& a, int device, cudaStream_t s, char* err, int errlen);
struct AttnBwdArgs {
  AttnArgs f;
  const void* dout;  // bf16 [B,S,Hq,hd], row stride ld_do
  long ld_do;
  void* dq;          // bf16 outputs, same layouts as q/k/v
  void* dk;
  void* dv;
  long ld_dq, ld_dk, ld_dv;
  float* dq_accum;   // fp32 scratch [B, S, Hq, hd] (zeroed by the launcher)
  float* delta;      // fp32 scratch [B, Hq, S]
};
int attention_bwd(const AttnBwdArgs& a, int device, cudaStream_t s, char* err, int errlen);

}  // namespace mt

// Allocation-free attention backward (defined in attention.cu; no counterpart in
// the reference).  For callers that cannot call cudaMalloc -- a host framework
// that owns every device allocation, code that must not risk an allocation's
// device synchronisation, plain C callers without a caching allocator.  Its dQ
// accumulator and delta rows live in one static 16 MiB device array per GPU:
// larger problems are rejected, the first call on a device (before any stream
// capture) looks up the array's address, and calls overlapping on the GPU race
// on the array.  Pointers must be non-NULL and 16-byte aligned (lse 4-byte).
// Returns 0, or non-zero with a message in err.
extern "C" int mt_attention_bwd_noalloc(const void* dout, long ld_do, const void* q, long ld_q, const void* k,
                                        long ld_k, const void* v, long ld_v, const void* o, long ld_o,
                                        const float* lse, void* dq, long ld_dq, void* dk, long ld_dk, void* dv,
                                        long ld_dv, int B, int S, int Hq, int Hk, int hd, float scale, int causal,
                                        cudaStream_t stream, uint32_t* device_status, char* err, int errlen);

// Reads and clears the status word that mt_attention_bwd_noalloc's kernels
// report a bounded-wait timeout into when they are given no device_status
// (current device; synchronous four-byte copies, no allocation).
extern "C" int mt_attention_noalloc_status(uint32_t* out, char* err, int errlen);
