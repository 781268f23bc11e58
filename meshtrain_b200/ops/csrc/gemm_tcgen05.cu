// gemm_tcgen05.cu -- persistent, warp-specialised bf16 GEMM for sm_100a.
//
//   D[M,N] = epilogue( A[M,K] * B[N,K]^T )      (fp32 accumulation in TMEM)
//
// A and B may each be K-major (row-major [rows, K]) or MN-major (row-major
// [K, rows]); that covers every linear-layer GEMM without a transpose copy:
//   forward  y  = x  W^T : A = x  (K-major),  B = W (K-major)
//   dgrad    dx = dy W   : A = dy (K-major),  B = W (MN-major, W is [K=out, N=in])
//   wgrad    dW += dy^T x: A = dy (MN-major), B = x (MN-major)
//
// Roles inside one CTA (192 threads, one CTA per SM, persistent over tiles):
//   warp 0      : TMA producer, fills a STAGES-deep ring of A/B k-blocks
//   warp 1      : allocates TMEM; one thread issues tcgen05.mma (128 x BN x 16)
//   warps 2..5  : epilogue, tcgen05.ld the accumulator (each warp owns the 32
//                 TMEM lanes its warp id allows), fuse bias / GELU / residual /
//                 dGELU / SwiGLU / fp32 accumulate, store to global.
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of tile i overlaps the MMAs of tile i+1.
//
// Replaces the cuBLAS GEMMs behind nn.Linear in the reference model
// (models/tiny_transformer.py:37-41, runtime/stage.py:28-36 via autograd).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "mt_api.h"
#include "sm100.cuh"

namespace mt {

enum Epi : int {
  kEpiBF16 = 0,     // D = acc (+ bias)                          bf16
  kEpiGelu = 1,     // H = acc + bias -> D2 = H, D = gelu(H)     bf16, bf16
  kEpiResid = 2,    // D = acc (+ bias) + R                      bf16
  kEpiDGelu = 3,    // D = acc * gelu'(R)                        bf16
  kEpiF32 = 4,      // D = beta * D + acc (+ bias)               fp32
  kEpiSwiGLU = 5,   // per 32 columns [16 gate | 16 up]: D2 = raw, D = silu(g) * u
};

struct GemmParams {  // device-side view of a GemmArgs
  int M, N, K;
  void* D;
  long ldd;
  void* D2;
  long ldd2;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* R;
  long ldr;
  float beta;
  int splits;        // split-K factor (fp32 epilogue with beta == 1 only)
  int kb_per_split;  // k-blocks per split
  uint32_t* status;
};

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kEpiWarps = 8;                   // two warpgroups split each tile's columns
constexpr int kThreads = 64 + 32 * kEpiWarps;  // TMA warp + MMA warp + epilogue

__device__ __forceinline__ void tile_coords(int tile, int m_tiles, int n_tiles, int& mb, int& nb) {
  // Group 16 M-blocks together so consecutive CTAs share B tiles in L2.
  constexpr int G = 16;
  const int group_size = G * n_tiles;
  const int group = tile / group_size;
  const int first_m = group * G;
  const int gm = min(m_tiles - first_m, G);
  const int local = tile - group * group_size;
  mb = first_m + local % gm;
  nb = local / gm;
}

// Epilogue math of one 32-column chunk of one row (EPI other than SwiGLU): bias
// (fp32 accumulate: lead split only), then GELU (the rounded pre-activation is
// returned packed in hw), residual add or GELU gradient.  v holds the outputs.
template <int EPI>
__device__ __forceinline__ void epi_apply(const GemmParams& p, int row, int col0, float* v, bool lead_split,
                                          uint32_t* hw) {
  const bool full = (col0 + 32 <= p.N);
  if (p.bias && (EPI != kEpiF32 || lead_split)) {
    if (full && ((reinterpret_cast<uintptr_t>(p.bias) & 15) == 0)) {
      // the 32 bias values of this chunk: four 16-byte loads, the same for every row (L1 hits)
      const uint4* b4 = reinterpret_cast<const uint4*>(p.bias + col0);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 q = b4[i];
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(w[j]);
          v[8 * i + 2 * j] += f.x;
          v[8 * i + 2 * j + 1] += f.y;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < p.N) v[i] += __bfloat162float(p.bias[col0 + i]);
    }
  }
  if constexpr (EPI == kEpiGelu) {
    // keep the rounded pre-activation for backward; GELU of the rounded value
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      hw[i >> 1] = pack_bf16x2(v[i], v[i + 1]);
      const float2 hr = unpack_bf16x2(hw[i >> 1]);
      v[i] = gelu_erf(hr.x);
      v[i + 1] = gelu_erf(hr.y);
    }
  } else if constexpr (EPI == kEpiResid || EPI == kEpiDGelu) {
    const __nv_bfloat16* r = p.R + (long)row * p.ldr + col0;
    if (full && ((p.ldr & 7) == 0)) {
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 q = *reinterpret_cast<const uint4*>(r + i);
        uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = unpack_bf16x2(w[j]);
          if constexpr (EPI == kEpiResid) {
            v[i + 2 * j] += f.x; v[i + 2 * j + 1] += f.y;
          } else {
            v[i + 2 * j] *= gelu_erf_grad(f.x); v[i + 2 * j + 1] *= gelu_erf_grad(f.y);
          }
        }
      }
    } else {
      for (int i = 0; i < 32; ++i) {
        if (col0 + i < p.N) {
          const float f = __bfloat162float(r[i]);
          if constexpr (EPI == kEpiResid) v[i] += f; else v[i] *= gelu_erf_grad(f);
        }
      }
    }
  }
}

// Epilogue of one 32-column chunk of one row written straight to global memory.
template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, int row, int col0, float* v, bool lead_split) {
  if (row >= p.M) return;
  const bool full = (col0 + 32 <= p.N);
  if constexpr (EPI == kEpiF32) {
    float* d = reinterpret_cast<float*>(p.D) + (long)row * p.ldd + col0;
    epi_apply<EPI>(p, row, col0, v, lead_split, nullptr);
    if (p.beta == 1.f) {
      // accumulate with fire-and-forget reductions: no read round trip, and
      // split-K partial products can land in any order
      if (full && ((p.ldd & 3) == 0)) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          atomicAdd(reinterpret_cast<float4*>(d + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
      } else {
        for (int i = 0; i < 32; ++i)
          if (col0 + i < p.N) atomicAdd(d + i, v[i]);
      }
      return;
    }
    if (full && ((p.ldd & 3) == 0)) {
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        float4 o = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        if (p.beta != 0.f) {
          float4 c = *reinterpret_cast<const float4*>(d + i);
          o.x += p.beta * c.x; o.y += p.beta * c.y; o.z += p.beta * c.z; o.w += p.beta * c.w;
        }
        *reinterpret_cast<float4*>(d + i) = o;
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < p.N) d[i] = v[i] + (p.beta != 0.f ? p.beta * d[i] : 0.f);
    }
    return;
  } else if constexpr (EPI == kEpiSwiGLU) {
    // 16 gate + 16 up columns -> 16 outputs at feature col0/2.
    __nv_bfloat16* raw = reinterpret_cast<__nv_bfloat16*>(p.D2) + (long)row * p.ldd2 + col0;
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.D) + (long)row * p.ldd + col0 / 2;
    uint32_t rw[16], ow[8];
#pragma unroll
    for (int i = 0; i < 16; ++i) rw[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // round the saved pre-activations first so backward sees the same values
      float2 g = unpack_bf16x2(pack_bf16x2(v[2 * i], v[2 * i + 1]));
      float2 u = unpack_bf16x2(pack_bf16x2(v[16 + 2 * i], v[16 + 2 * i + 1]));
      ow[i] = pack_bf16x2(silu(g.x) * u.x, silu(g.y) * u.y);
    }
    if (full) {
      uint4* r4 = reinterpret_cast<uint4*>(raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) r4[i] = make_uint4(rw[4 * i], rw[4 * i + 1], rw[4 * i + 2], rw[4 * i + 3]);
      uint4* o4 = reinterpret_cast<uint4*>(out);
#pragma unroll
      for (int i = 0; i < 2; ++i) o4[i] = make_uint4(ow[4 * i], ow[4 * i + 1], ow[4 * i + 2], ow[4 * i + 3]);
    }
    return;
  } else {
    __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(p.D) + (long)row * p.ldd + col0;
    uint32_t hw[16];
    epi_apply<EPI>(p, row, col0, v, lead_split, hw);
    if constexpr (EPI == kEpiGelu) {
      __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(p.D2) + (long)row * p.ldd2 + col0;
      if (full && ((p.ldd2 & 7) == 0)) {
        uint4* h4 = reinterpret_cast<uint4*>(h);
#pragma unroll
        for (int i = 0; i < 4; ++i) h4[i] = make_uint4(hw[4 * i], hw[4 * i + 1], hw[4 * i + 2], hw[4 * i + 3]);
      } else {
        for (int i = 0; i < 32; ++i)
          if (col0 + i < p.N) h[i] = __ushort_as_bfloat16((unsigned short)((hw[i >> 1] >> (16 * (i & 1))) & 0xFFFF));
      }
    }
    if (full && ((p.ldd & 7) == 0)) {
      uint4* d4 = reinterpret_cast<uint4*>(d);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        d4[i] = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                           pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < p.N) d[i] = __float2bfloat16_rn(v[i]);
    }
  }
}

// ---- staged epilogue: rows -> swizzled shared-memory tiles -> TMA bulk stores
// Each epilogue warp owns 32 rows of the tile; per 32-column chunk it writes its
// [32 x 32] block into one of two staging buffers and one lane issues the bulk
// tensor store (bf16) or bulk reduce-add (fp32 accumulate).  The TMA clips rows
// and columns outside the output, so partial tiles need no special casing.
constexpr int kStgBuffers = 2;

// 32 bf16 (16 packed words) of row r of a [32 rows x 64 B] tile, 64-byte swizzle.
__device__ __forceinline__ void stage_row_bf16_sw64(uint8_t* tile, int r, const uint32_t* w) {
  uint8_t* line = tile + r * 64;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    *reinterpret_cast<uint4*>(line + ((c ^ ((r >> 1) & 3)) << 4)) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

// 32 fp32 of row r of a [32 rows x 128 B] tile, 128-byte swizzle.
__device__ __forceinline__ void stage_row_f32_sw128(uint8_t* tile, int r, const float* v) {
  uint8_t* line = tile + r * 128;
#pragma unroll
  for (int u = 0; u < 8; ++u)
    *reinterpret_cast<float4*>(line + ((u ^ (r & 7)) << 4)) = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  // x 16-byte aligned for fp32 outputs (bf16 ones need a multiple of 8); no negative start
  if (!MT_CHECK((x & 3) == 0 && x >= 0 && y >= 0, kErrCheckTma)) return;
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int x, int y) {
  // x 16-byte aligned for fp32 outputs (bf16 ones need a multiple of 8); no negative start
  if (!MT_CHECK((x & 3) == 0 && x >= 0 && y >= 0, kErrCheckTma)) return;
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// at most kStgBuffers-1 bulk groups may still be reading shared memory
__device__ __forceinline__ void bulk_wait_read_stg() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kStgBuffers - 1) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

template <int EPI>
struct StageCfg {
  // bytes of one staging buffer of one warp: the output block, plus the GELU pre-activation block
  static constexpr int kBuf = EPI == kEpiF32 ? 32 * 128 : (EPI == kEpiGelu ? 2 : 1) * 32 * 64;
  static constexpr int kBytes = kEpiWarps * kStgBuffers * kBuf;
};

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const GemmParams p) {
  constexpr int A_BYTES = kBM * kBK * 2;
  constexpr int B_BYTES = BN * kBK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;  // double-buffered fp32 accumulator
  static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of two");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((base_u32 + 1023u) & ~1023u) - base_u32);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tslot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  const int m_tiles = (p.M + kBM - 1) / kBM;
  const int n_tiles = (p.N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (p.K + kBK - 1) / kBK;
  // Work unit u = (split, tile): consecutive units share a K range, so CTAs that
  // run together read the same A/B k-slices from L2.
  const int num_units = num_tiles * p.splits;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed_mask = 0, armed_parity = 0;
      for (int u = blockIdx.x; u < num_units && !*abort_flag; u += gridDim.x) {
        const int tile = u % num_tiles, split = u / num_tiles;
        int mb, nb;
        tile_coords(tile, m_tiles, n_tiles, mb, nb);
        const int kb0 = split * p.kb_per_split, kb1 = min(k_blocks, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status, kErrWaitEmpty)) goto producer_done;
          mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
          armed_mask |= 1u << stage;
          armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          if constexpr (!A_MN) {
            tma_load_2d(a_dst, &tmA, &full[stage], kb * kBK, mb * kBM);
          } else {
#pragma unroll
            for (int c = 0; c < kBM / 64; ++c) tma_load_2d(a_dst + c * 8192, &tmA, &full[stage], mb * kBM + c * 64, kb * kBK);
          }
          if constexpr (!B_MN) {
            tma_load_2d(b_dst, &tmB, &full[stage], kb * kBK, nb * BN);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_2d(b_dst + c * 8192, &tmB, &full[stage], nb * BN + c * 64, kb * kBK);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:
      // Never leave the CTA with bulk copies still landing in shared memory.
      for (int s = 0; s < STAGES; ++s) {
        if (armed_mask & (1u << s)) {
          volatile int no_abort = 0;
          mbar_wait(&full[s], (armed_parity >> s) & 1u, &no_abort, p.status, kErrWaitFull);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc = idesc_bf16_f32(kBM, BN, A_MN, B_MN);
      const uint64_t a_desc0 = A_MN ? desc_sw128(smem_u32(sA), 8192, 1024) : desc_sw128(smem_u32(sA), 16, 1024);
      const uint64_t b_desc0 = B_MN ? desc_sw128(smem_u32(sB), 8192, 1024) : desc_sw128(smem_u32(sB), 16, 1024);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int u = blockIdx.x; u < num_units && !*abort_flag; u += gridDim.x) {
        const int split = u / num_tiles;
        const int kb0 = split * p.kb_per_split, kb1 = min(k_blocks, kb0 + p.kb_per_split);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.status, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tbase + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a_st = desc_add(a_desc0, (uint32_t)(stage * A_BYTES));
          const uint64_t b_st = desc_add(b_desc0, (uint32_t)(stage * B_BYTES));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_bf16_ss(d_tmem, desc_add(a_st, A_MN ? kk * 2048 : kk * 32), desc_add(b_st, B_MN ? kk * 2048 : kk * 32),
                         idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
          umma_commit(&empty[stage]);  // frees the smem stage when these MMAs retire
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // Wait (bounded) for every MMA this thread issued before TMEM is freed.
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, p.status, kErrWaitAccum);
    }
    __syncwarp();
  } else {
    // Epilogue: warp w may touch TMEM lanes [32*(w%4), 32*(w%4)+32); the two
    // warpgroups take the left and right halves of the tile's columns.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
      const int tile = u % num_tiles;
      const bool lead_split = u < num_tiles;
      int mb, nb;
      tile_coords(tile, m_tiles, n_tiles, mb, nb);
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status, kErrWaitAccum) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const int row = mb * kBM + q * 32 + lane;
      const uint32_t t_row = tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
        float v[32];
        tmem_ld_32x32b_x32(t_row + c * 32, v);
        const int col0 = nb * BN + c * 32;
        if (col0 < p.N) epilogue_chunk<EPI>(p, row, col0, v, lead_split);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}


// CTA-pair variant: a cluster of two CTAs computes one 256 x BN tile with
// tcgen05.mma.cta_group::2 (M = 256).  Each CTA loads its own 128 rows of A and
// BN/2 rows of B into its own shared memory, so per SM the operand traffic per
// FLOP is two thirds of the single-CTA 128 x BN tile.  Both CTAs' loads count
// their bytes on the even CTA's `full` barrier (which expects both halves); the
// even CTA issues the MMAs, whose commits free the stage in both CTAs (one
// commit per CTA) and signal both CTAs' accumulator barriers; both epilogues
// arrive on the even CTA's tempty.  A cluster barrier at the end keeps either
// CTA resident until the pair's MMAs, which read both CTAs' shared memory, are done.
// STAGED: the epilogue writes through shared-memory staging tiles and TMA bulk
// stores / reduce-adds (tmD, tmD2) instead of per-thread global stores.
template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, bool STAGED>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmD2,
                     const GemmParams p) {
  constexpr int BNH = BN / 2;
  constexpr int A_BYTES = kBM * kBK * 2;
  constexpr int B_BYTES = BNH * kBK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of two");
  constexpr int STG_BYTES = STAGED ? StageCfg<EPI>::kBytes : 0;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((base_u32 + 1023u) & ~1023u) - base_u32);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sStg = sB + STAGES * B_BYTES;  // 1024-byte aligned: stage sizes are multiples of 1 KB
  uint64_t* full = reinterpret_cast<uint64_t*>(sStg + STG_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool even = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tslot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised, TMEM allocated on both SMs
  tc_fence_after();
  const uint32_t tbase = *tslot;

  const int m_tiles = (p.M + 2 * kBM - 1) / (2 * kBM);
  const int n_tiles = (p.N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (p.K + kBK - 1) / kBK;
  const int num_units = num_tiles * p.splits;
  const int cid = (int)(blockIdx.x >> 1), ncl = (int)(gridDim.x >> 1);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed_mask = 0, armed_parity = 0;
      for (int u = cid; u < num_units && !*abort_flag; u += ncl) {
        const int tile = u % num_tiles, split = u / num_tiles;
        int mb, nb;
        tile_coords(tile, m_tiles, n_tiles, mb, nb);
        const int m0 = mb * 2 * kBM + (int)rank * kBM, n0 = nb * BN + (int)rank * BNH;
        const int kb0 = split * p.kb_per_split, kb1 = min(k_blocks, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status, kErrWaitEmpty)) goto pair_producer_done;
          if (even) {  // the even CTA's barrier counts both CTAs' bytes
            mbar_arrive_expect_tx(&full[stage], 2 * (A_BYTES + B_BYTES));
            armed_mask |= 1u << stage;
            armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          }
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          if constexpr (!A_MN) {
            tma_load_2d_pair(a_dst, &tmA, &full[stage], kb * kBK, m0);
          } else {
#pragma unroll
            for (int c = 0; c < kBM / 64; ++c)
              tma_load_2d_pair(a_dst + c * 8192, &tmA, &full[stage], m0 + c * 64, kb * kBK);
          }
          if constexpr (!B_MN) {
            tma_load_2d_pair(b_dst, &tmB, &full[stage], kb * kBK, n0);
          } else {
#pragma unroll
            for (int c = 0; c < BNH / 64; ++c)
              tma_load_2d_pair(b_dst + c * 8192, &tmB, &full[stage], n0 + c * 64, kb * kBK);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    pair_producer_done:
      for (int s = 0; s < STAGES; ++s) {
        if (armed_mask & (1u << s)) {
          volatile int no_abort = 0;
          mbar_wait(&full[s], (armed_parity >> s) & 1u, &no_abort, p.status, kErrWaitFull);
        }
      }
    }
  } else if (warp == 1) {
    if (even && elect_one()) {
      const uint32_t idesc = idesc_bf16_f32(2 * kBM, BN, A_MN, B_MN);
      const uint64_t a_desc0 = A_MN ? desc_sw128(smem_u32(sA), 8192, 1024) : desc_sw128(smem_u32(sA), 16, 1024);
      const uint64_t b_desc0 = B_MN ? desc_sw128(smem_u32(sB), 8192, 1024) : desc_sw128(smem_u32(sB), 16, 1024);
      const uint32_t empty_c0 = cluster_addr(&empty[0], 0), empty_c1 = cluster_addr(&empty[0], 1);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int u = cid; u < num_units && !*abort_flag; u += ncl) {
        const int split = u / num_tiles;
        const int kb0 = split * p.kb_per_split, kb1 = min(k_blocks, kb0 + p.kb_per_split);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.status, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tbase + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a_st = desc_add(a_desc0, (uint32_t)(stage * A_BYTES));
          const uint64_t b_st = desc_add(b_desc0, (uint32_t)(stage * B_BYTES));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_bf16_ss_pair(d_tmem, desc_add(a_st, A_MN ? kk * 2048 : kk * 32),
                              desc_add(b_st, B_MN ? kk * 2048 : kk * 32), idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
          umma_commit_pair(empty_c0 + 8u * (uint32_t)stage);  // frees this stage in both CTAs once the MMAs retire
          umma_commit_pair(empty_c1 + 8u * (uint32_t)stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(cluster_addr(&tfull[acc], 0));
        umma_commit_pair(cluster_addr(&tfull[acc], 1));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      umma_commit_pair(cluster_addr(drain, 0));
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, p.status, kErrWaitAccum);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* stg = sStg + (warp - 2) * kStgBuffers * (STAGED ? StageCfg<EPI>::kBuf : 0);
    int sbuf = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = cid; u < num_units; u += ncl) {
      const int tile = u % num_tiles;
      const bool lead_split = u < num_tiles;
      int mb, nb;
      tile_coords(tile, m_tiles, n_tiles, mb, nb);
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status, kErrWaitAccum) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const int row0 = mb * 2 * kBM + (int)rank * kBM + q * 32;
      const int row = row0 + lane;
      const uint32_t t_row = tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
        float v[32];
        tmem_ld_32x32b_x32(t_row + c * 32, v);
        const int col0 = nb * BN + c * 32;
        if (col0 >= p.N) continue;
        if constexpr (STAGED) {
          uint32_t hw[16];
          if (row < p.M) epi_apply<EPI>(p, row, col0, v, lead_split, hw);
          uint8_t* buf = stg + sbuf * StageCfg<EPI>::kBuf;
          if (lane == 0) bulk_wait_read_stg();  // the store that last used this buffer has read it
          __syncwarp();
          if constexpr (EPI == kEpiF32) {
            stage_row_f32_sw128(buf, lane, v);
          } else {
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
            stage_row_bf16_sw64(buf, lane, w);
            if constexpr (EPI == kEpiGelu) stage_row_bf16_sw64(buf + 32 * 64, lane, hw);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if constexpr (EPI == kEpiF32) {
              if (p.beta == 1.f) tma_reduce_add_2d(&tmD, buf, col0, row0);
              else tma_store_2d(&tmD, buf, col0, row0);
            } else {
              tma_store_2d(&tmD, buf, col0, row0);
              if constexpr (EPI == kEpiGelu) tma_store_2d(&tmD2, buf + 32 * 64, col0, row0);
            }
            bulk_commit();
          }
          sbuf ^= 1;
        } else {
          epilogue_chunk<EPI>(p, row, col0, v, lead_split);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_addr(&tempty[acc], 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (STAGED && lane == 0) bulk_wait_all();  // every bulk store has completed before the CTA retires
  }

  tc_fence_before();
  cluster_sync();  // the pair's MMAs and remote arrivals are over before either CTA leaves
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// bf16 2-D tensor map over a row-major matrix [outer, inner] with leading dim
// ld (elements); box {64 inner, box_outer}; 128-byte swizzle; zero fill.
static bool make_map(CUtensorMap* m, const void* ptr, long inner, long outer, long ld, int box_outer) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1u, 1u};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms(int dev) {
  static int cached[64] = {0};
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
static int launch(const GemmArgs& g, const GemmParams& p, int dev, cudaStream_t stream, char* err, int errlen) {
  constexpr int smem = STAGES * (kBM * kBK * 2 + BN * kBK * 2) + 1024 + 256;
  CUtensorMap ta, tb;
  const bool ok_a = A_MN ? make_map(&ta, g.a, g.M, g.K, g.lda, 64) : make_map(&ta, g.a, g.K, g.M, g.lda, kBM);
  const bool ok_b = B_MN ? make_map(&tb, g.b, g.N, g.K, g.ldb, 64) : make_map(&tb, g.b, g.K, g.N, g.ldb, BN);
  if (!ok_a || !ok_b) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled failed (M=%d N=%d K=%d lda=%ld ldb=%ld)", g.M, g.N, g.K, g.lda, g.ldb);
    return -1;
  }
  auto kern = gemm_tcgen05_kernel<BN, STAGES, A_MN, B_MN, EPI>;
  static bool attr_set[64] = {false};
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int tiles = ((g.M + kBM - 1) / kBM) * ((g.N + BN - 1) / BN) * p.splits;
  const int grid = std::max(1, std::min(tiles, num_sms(dev)));
  kern<<<grid, kThreads, smem, stream>>>(ta, tb, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(err, errlen, "gemm launch failed: %s", cudaGetErrorString(e));
    return (int)e;
  }
  return 0;
}

// Output map of the staged epilogue: [outer, inner] row-major with leading dim ld,
// box {32 inner, 32 outer}; bf16 with 64-byte swizzle, fp32 with 128-byte swizzle.
static bool make_out_map(CUtensorMap* m, const void* ptr, bool f32, long inner, long outer, long ld) {
  auto fn = encode_fn();
  if (!fn) return false;
  const int es = f32 ? 4 : 2;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
  cuuint32_t box[2] = {32u, 32u};
  cuuint32_t estr[2] = {1u, 1u};
  return fn(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The staged epilogue applies when the outputs suit bulk tensor stores (16-byte
// aligned base and row pitch) and the epilogue is a plain store, a store pair
// (GELU) or an fp32 store / accumulate.  MT_GEMM_STAGED=0 switches it off.
static bool staged_epilogue_ok(const GemmArgs& g) {
  static int env = -1;
  if (env < 0) {
    const char* e = getenv("MT_GEMM_STAGED");
    env = (e && e[0] == '0') ? 0 : 1;
  }
  if (!env || g.epi == kEpiSwiGLU) return false;
  const bool f32 = g.epi == kEpiF32;
  const int es = f32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(g.d) & 15) || ((g.ldd * es) & 15)) return false;
  if (f32 && g.beta != 0.f && g.beta != 1.f) return false;
  if (g.epi == kEpiGelu && ((reinterpret_cast<uintptr_t>(g.d2) & 15) || ((g.ldd2 * 2) & 15))) return false;
  return true;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, bool STAGED>
static int launch_pair(const GemmArgs& g, const GemmParams& p, int dev, cudaStream_t stream, char* err,
                       int errlen) {
  constexpr int smem =
      STAGES * (kBM * kBK * 2 + (BN / 2) * kBK * 2) + (STAGED ? StageCfg<EPI>::kBytes : 0) + 1024 + 256;
  static_assert(smem <= 232448, "shared memory per CTA exceeds 227 KB");
  CUtensorMap ta, tb, td, td2;
  const bool ok_a = A_MN ? make_map(&ta, g.a, g.M, g.K, g.lda, 64) : make_map(&ta, g.a, g.K, g.M, g.lda, kBM);
  const bool ok_b = B_MN ? make_map(&tb, g.b, g.N, g.K, g.ldb, 64) : make_map(&tb, g.b, g.K, g.N, g.ldb, BN / 2);
  bool ok_d = true;
  memset(&td, 0, sizeof(td));
  memset(&td2, 0, sizeof(td2));
  if (STAGED) {
    ok_d = make_out_map(&td, g.d, EPI == kEpiF32, g.N, g.M, g.ldd);
    if (EPI == kEpiGelu) ok_d = ok_d && make_out_map(&td2, g.d2, false, g.N, g.M, g.ldd2);
  }
  if (!ok_a || !ok_b || !ok_d) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled failed (M=%d N=%d K=%d lda=%ld ldb=%ld)", g.M, g.N, g.K, g.lda, g.ldb);
    return -1;
  }
  auto kern = gemm_pair_kernel<BN, STAGES, A_MN, B_MN, EPI, STAGED>;
  static bool attr_set[64] = {false};
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const long units = (long)((g.M + 2 * kBM - 1) / (2 * kBM)) * ((g.N + BN - 1) / BN) * p.splits;
  const int clusters = (int)std::max(1L, std::min(units, (long)(num_sms(dev) / 2)));
  kern<<<2 * clusters, kThreads, smem, stream>>>(ta, tb, td, td2, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(err, errlen, "gemm (CTA pair) launch failed: %s", cudaGetErrorString(e));
    return (int)e;
  }
  return 0;
}

// Fraction of the persistent grid doing useful work in the last wave.
static double wave_efficiency(long units, int sms) {
  const long waves = (units + sms - 1) / sms;
  return (double)units / (double)(waves * sms);
}

struct TilePlan {
  bool pair;  // 256-row tiles on a CTA pair (cta_group::2) instead of 128-row tiles on one CTA
  int bn;
  int splits;
  int kb_per_split;
};

// CTA pairs can be switched off with MT_GEMM_PAIR=0 (single-CTA kernels only).
static bool pair_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("MT_GEMM_PAIR");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// Pick the tile shape and, for accumulating fp32 epilogues, a split-K factor so
// the persistent grid has few idle SMs in its last wave.  Relative throughput of
// the shapes, measured on the linear-layer GEMMs of the 0.48B GPT (M=8192,
// N 1280..5120, K 1280..8192) on one B200: pair 256x256 1.0, single 128x256
// 0.90, single 128x128 0.70, pair 256x128 0.60 -- the narrow tiles move too many
// operand bytes through shared memory per FLOP, which outweighs their finer
// last wave.
// MT_GEMM_SHAPE=pair256|pair128|single256|single128 forces one tile shape (benchmarking).
static int forced_shape() {
  static int v = -2;
  if (v == -2) {
    const char* e = getenv("MT_GEMM_SHAPE");
    v = -1;
    if (e) {
      const char* names[4] = {"pair256", "pair128", "single256", "single128"};
      for (int i = 0; i < 4; ++i)
        if (strcmp(e, names[i]) == 0) v = i;
    }
  }
  return v;
}

static TilePlan plan_tiles(const GemmArgs& g, int sms, bool can_split) {
  const int k_blocks = (g.K + kBK - 1) / kBK;
  TilePlan best{false, 256, 1, k_blocks};
  double best_score = -1.0;
  struct Shape { bool pair; int bn; double rate; };
  const Shape shapes[4] = {{true, 256, 1.0}, {true, 128, 0.60}, {false, 256, 0.90}, {false, 128, 0.70}};
  const int forced = forced_shape();
  for (int si = 0; si < 4; ++si) {
    const Shape& sh = shapes[si];
    if (forced >= 0 && si != forced) continue;
    if (sh.pair && (!pair_enabled() || g.M < 2 * kBM) && forced < 0) continue;
    if (sh.bn == 256 && g.N < 256) continue;
    const int rows = sh.pair ? 2 * kBM : kBM;
    const long tiles = (long)((g.M + rows - 1) / rows) * ((g.N + sh.bn - 1) / sh.bn);
    const int slots = sh.pair ? sms / 2 : sms;
    const int max_split = can_split ? std::max(1, std::min(16, k_blocks / 8)) : 1;
    for (int sp = 1; sp <= max_split; ++sp) {
      const int kpb = (k_blocks + sp - 1) / sp;
      const int eff_sp = (k_blocks + kpb - 1) / kpb;  // no empty splits
      const double score = wave_efficiency(tiles * eff_sp, slots) * sh.rate * (1.0 - 0.01 * (eff_sp - 1));
      if (score > best_score + 1e-9) {
        best_score = score;
        best = TilePlan{sh.pair, sh.bn, eff_sp, kpb};
      }
    }
  }
  return best;
}

template <bool A_MN, bool B_MN, int EPI>
static int dispatch_bn(const GemmArgs& g, GemmParams p, int dev, cudaStream_t s, char* err, int errlen) {
  const bool can_split = (EPI == kEpiF32) && g.beta == 1.f;
  const TilePlan t = plan_tiles(g, num_sms(dev), can_split);
  p.splits = t.splits;
  p.kb_per_split = t.kb_per_split;
  if (t.pair) {
    if (t.bn == 256) {
      if constexpr (EPI != kEpiSwiGLU) {
        // staging takes shared memory from the operand ring: 6 stages for one bf16
        // output, 5 for two outputs (GELU) or fp32
        constexpr int ST = (EPI == kEpiGelu || EPI == kEpiF32) ? 5 : 6;
        if (staged_epilogue_ok(g)) return launch_pair<256, ST, A_MN, B_MN, EPI, true>(g, p, dev, s, err, errlen);
      }
      return launch_pair<256, 7, A_MN, B_MN, EPI, false>(g, p, dev, s, err, errlen);
    }
    return launch_pair<128, 9, A_MN, B_MN, EPI, false>(g, p, dev, s, err, errlen);
  }
  if (t.bn == 256) return launch<256, 4, A_MN, B_MN, EPI>(g, p, dev, s, err, errlen);
  return launch<128, 6, A_MN, B_MN, EPI>(g, p, dev, s, err, errlen);
}

static uint32_t* g_status[64] = {nullptr};
static std::mutex g_status_mu;

uint32_t* device_status(int dev) {
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!g_status[dev]) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(dev);
    if (cudaMalloc(&g_status[dev], 64) == cudaSuccess) cudaMemset(g_status[dev], 0, 64);
    else g_status[dev] = nullptr;
    cudaSetDevice(prev);
  }
  return g_status[dev];
}

// Debug-check words of every translation unit (each registers its reader at load).
static std::vector<uint32_t (*)()>& check_readers() {
  static std::vector<uint32_t (*)()> readers;
  return readers;
}
void register_check_reader(uint32_t (*reader)()) { check_readers().push_back(reader); }
uint32_t read_and_clear_checks() {
  uint32_t flags = 0;
  for (auto reader : check_readers()) flags |= reader();
  return flags;
}
bool debug_checks_built() {
#ifdef MT_DEBUG_CHECKS
  return true;
#else
  return false;
#endif
}

uint32_t read_and_clear_status(int dev) {
  uint32_t* w = device_status(dev);
  if (!w) return 0xFFFFFFFFu;
  uint32_t h = 0;
  cudaMemcpy(&h, w, 4, cudaMemcpyDeviceToHost);
  cudaMemset(w, 0, 4);
  return h;
}

int gemm_launch(const GemmArgs& g, int dev, cudaStream_t s, char* err, int errlen) {
  if (g.M <= 0 || g.N <= 0) return 0;
  GemmParams p{};
  p.M = g.M;
  p.N = g.N;
  p.K = g.K;
  p.D = g.d;
  p.ldd = g.ldd;
  p.D2 = g.d2;
  p.ldd2 = g.ldd2;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(g.bias);
  p.R = reinterpret_cast<const __nv_bfloat16*>(g.aux);
  p.ldr = g.ldaux;
  p.beta = g.beta;
  p.status = device_status(dev);
#define MT_CASE(AM, BMJ, E) \
  if (g.a_mn == AM && g.b_mn == BMJ && g.epi == E) return dispatch_bn<AM, BMJ, E>(g, p, dev, s, err, errlen);
  MT_CASE(false, false, kEpiBF16)
  MT_CASE(false, false, kEpiGelu)
  MT_CASE(false, false, kEpiResid)
  MT_CASE(false, false, kEpiSwiGLU)
  MT_CASE(false, false, kEpiF32)
  MT_CASE(false, true, kEpiBF16)
  MT_CASE(false, true, kEpiDGelu)
  MT_CASE(false, true, kEpiF32)
  MT_CASE(true, true, kEpiF32)
  MT_CASE(true, true, kEpiBF16)
  MT_CASE(true, false, kEpiF32)
#undef MT_CASE
  snprintf(err, errlen, "gemm: unsupported combination a_mn=%d b_mn=%d epi=%d", (int)g.a_mn, (int)g.b_mn, g.epi);
  return -2;
}

}  // namespace mt
