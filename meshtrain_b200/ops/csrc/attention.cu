// attention.cu -- causal / GQA flash attention forward and backward on tcgen05.
//
// Layout: q [B, S, Hq, HD], k/v [B, S, Hk, HD] as rows of width ld (strided
// views into a packed QKV activation are fine), o [B, S, Hq, HD], lse [B, Hq, S]
// (natural-log logsumexp of the scaled scores).  HD is 64 or 128.  Tiles are
// 128 queries x 128 keys; a 3-D TMA map {cols, S, B} per tensor zero-fills rows
// past S, which the kernels mask.
//
// Forward (one CTA per (128-query tile, batch*head)):
//   warp 0     TMA: Q once, then K_j / V_j into separate smem rings
//   warp 1     one thread issues S_j = Q K_j^T (TMEM, double-buffered) and
//              O += P_j V_j (TMEM); Q and P_j are A operands read from TMEM, so
//              shared memory only carries K_j and V_j (V as an MN-major operand)
//   warps 2-5  softmax: thread i owns query row i (TMEM lane i): copies its Q
//              row into TMEM once, then per tile loads S_j, takes the row max,
//              writes P_j = 2^(s - m_ref) as bf16 into TMEM; O is rescaled in
//              TMEM only when the row maximum grows by more than 2^8
//
// Backward (one CTA per (128-key tile, batch*kv-head), looping over the query
// tiles and the q heads of the GQA group, so dK / dV accumulate in TMEM):
//   S^T = K Q^T, dP^T = V dO^T                      (TMEM)
//   P^T = exp2(S^T*c - lse2), dS^T = P^T (dP^T - D)  (softmax warps, -> smem)
//   dV += P^T dO, dK += dS^T Q                       (TMEM accumulators)
//   dQ  = dS K  -> fp32 atomics into a scratch dQ accumulator
// Every smem tile is reused as a K-major and as an MN-major operand by giving
// the tensor core a different descriptor, so nothing is transposed.
//
// Replaces F.scaled_dot_product_attention(is_causal=True) in the reference
// (models/tiny_transformer.py:47).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <type_traits>
#include <mutex>

#include "mt_api.h"
#include "sm100.cuh"

namespace mt {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kTile = 128;
constexpr int kChunkBytes = kTile * 128;  // 128 rows x 64 bf16 (one 128-byte swizzle column)

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  if (!MT_CHECK((x & 7) == 0, kErrCheckTma)) return;  // bf16 maps: x * 2 bytes must be 16-byte aligned
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}


// Store 32 bf16 values (one thread's row segment of 32 columns, column block c)
// into a K-major SW128 operand tile made of 64-column chunks of 128 rows.
__device__ __forceinline__ void store_row32_sw128(uint8_t* tile, int row, int c, const uint32_t* packed16) {
  uint8_t* chunk = tile + (c >> 1) * kChunkBytes + row * 128;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int unit = ((c & 1) << 2) + w;
    uint4 v = make_uint4(packed16[4 * w], packed16[4 * w + 1], packed16[4 * w + 2], packed16[4 * w + 3]);
    *reinterpret_cast<uint4*>(chunk + ((unit ^ (row & 7)) << 4)) = v;
  }
}

__device__ __forceinline__ bool wait_lane0(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                           uint32_t* status, uint32_t code) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, status, code) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Per-role timestamps of the backward pipeline (diagnostic builds only: compile
// with -DMT_ATTN_TRACE).  CTAs of batch-head 0 record clock64() at the pipeline
// events of each query-tile iteration into g_attn_trace[kt][it][event].
#ifdef MT_ATTN_TRACE
constexpr int kTrKt = 32, kTrIt = 64, kTrEv = 16;
__device__ unsigned long long g_attn_trace[kTrKt * kTrIt * kTrEv];
#define ATTN_TRACE(kt, it, ev)                                                                         \
  do {                                                                                                 \
    if (blockIdx.y == 0 && (kt) < kTrKt && (it) < kTrIt)                                                \
      g_attn_trace[((kt) * kTrIt + (it)) * kTrEv + (ev)] = (unsigned long long)clock64();              \
  } while (0)
#define ATTN_TRACE_T(tid, kt, it, ev) \
  do {                                \
    if (threadIdx.x == (tid)) ATTN_TRACE(kt, it, ev); \
  } while (0)
// backward: CTA 0 records the events of its global iteration g (g < kTrKt * kTrIt)
#define BWD_TRACE(g, ev)                                                                      \
  do {                                                                                        \
    if (blockIdx.x == 0 && (g) >= 0 && (g) < kTrKt * kTrIt)                                     \
      g_attn_trace[(long)(g) * kTrEv + (ev)] = (unsigned long long)clock64();                  \
  } while (0)
// forward (two-query-tile kernel): CTA (0, 0) records the events of its KV step j
#define FWD_TRACE(j, ev)                                                                      \
  do {                                                                                        \
    if (blockIdx.x == 0 && blockIdx.y == 0 && (j) >= 0 && (j) < kTrKt * kTrIt)                  \
      g_attn_trace[(long)(j) * kTrEv + (ev)] = (unsigned long long)clock64();                  \
  } while (0)
#else
#define FWD_TRACE(j, ev) \
  do {                   \
  } while (0)
#define BWD_TRACE(g, ev) \
  do {                   \
  } while (0)
#define ATTN_TRACE(kt, it, ev) \
  do {                         \
  } while (0)
#define ATTN_TRACE_T(tid, kt, it, ev) \
  do {                                \
  } while (0)
#endif

struct FwdParams {
  __nv_bfloat16* o;
  long ld_o;
  float* lse;
  int B, S, Hq, Hk;
  float scale_log2;
  int causal;
  uint32_t* status;
  int alternate;  // ping-pong kernel: hand the exponential phase from one warpgroup to the other
};

template <int HD, int ST>
struct FwdSmem {
  static constexpr int kQ = HD / 64 * kChunkBytes;  // Q staging (TMA -> smem -> TMEM)
  static constexpr int kKV = kQ;
  static constexpr int kBytes = kQ + 2 * ST * kKV;
};

// TMEM columns of the forward: S_j double-buffered, the running output O, the
// bf16 probabilities P_j and the bf16 query tile Q (the last two are the A
// operands of P V and Q K^T, packed two per column).
template <int HD>
struct FwdTmem {
  static constexpr uint32_t kS = 0;                 // 2 x 128
  static constexpr uint32_t kO = 256;               // HD
  static constexpr uint32_t kP = kO + HD;           // 64
  static constexpr uint32_t kQ = kP + 64;           // HD / 2
  static constexpr uint32_t kCols = 512;
  static_assert(kQ + HD / 2 <= kCols, "forward TMEM layout exceeds 512 columns");
};

// Lazy rescaling: P_j = 2^(s - m_ref) keeps the row's reference maximum m_ref
// until a new score exceeds it by more than 2^8, so O (in TMEM) is rescaled
// only then; P <= 256 loses nothing in bf16 and O / l is exact in fp32.
constexpr float kRescaleLog2 = 8.0f;

// Running maximum over 32 more columns with sm_100's three-input max: two
// independent chains of eight.
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float max32(const float* v, float m) {
  float r0 = m, r1 = -INFINITY;
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    r0 = max3f(r0, v[i], v[i + 1]);
    r1 = max3f(r1, v[i + 2], v[i + 3]);
  }
  return fmaxf(r0, r1);
}

// Row maximum of 128 columns: four independent chains of three-input maxima.
__device__ __forceinline__ float max128(const float* v) {
  const float a = max32(v, -INFINITY), b = max32(v + 32, -INFINITY);
  const float c = max32(v + 64, -INFINITY), d = max32(v + 96, -INFINITY);
  return fmaxf(fmaxf(a, b), fmaxf(c, d));
}

// Exponentials of the forward softmax for 32 columns of one row:
// P = 2^(s * sc - m) as bf16 pairs into pk, fp32 row sums into acc[4].  KPOLY of every 16 column pairs go through ex2_poly_x2 (FMA pipe), the
// rest through the special-function unit; KPOLY = 0 (masked tiles, where exact
// zeros are needed) uses the special-function unit only.
template <int KPOLY>
__device__ __forceinline__ void fwd_exp32(const float* v, float sc, float negm, uint32_t* pk, float* acc) {
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    float e0, e1;
    if (KPOLY > 0 && poly_pair<KPOLY>(q)) {
      f2unpack(ex2_poly_x2(fma_f32x2(f2pack(v[2 * q], v[2 * q + 1]), f2pack(sc, sc), f2pack(negm, negm))), e0, e1);
    } else {
      e0 = ex2_approx(fmaf(v[2 * q], sc, negm));
      e1 = ex2_approx(fmaf(v[2 * q + 1], sc, negm));
    }
    acc[q & 3] += e0 + e1;
    pk[q] = pack_bf16x2(e0, e1);
  }
}

// Share of the forward's exponentials on the FMA pipe (pairs of 16).
#ifndef MT_FWD_POLY_PAIRS
#define MT_FWD_POLY_PAIRS 6
#endif
constexpr int kFwdPolyPairs = MT_FWD_POLY_PAIRS;

template <int HD, int ST, int KP = kFwdPolyPairs>
__global__ void __launch_bounds__(192, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  using L = FwdSmem<HD, ST>;
  using T = FwdTmem<HD>;
  constexpr int NCH = HD / 64;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((base_u32 + 1023u) & ~1023u) - base_u32);
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + L::kQ;
  uint8_t* sV = sK + ST * L::kKV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + ST * L::kKV);
  uint64_t* q_full = bars;
  uint64_t* q_tmem = q_full + 1;
  uint64_t* k_full = q_tmem + 1;
  uint64_t* k_empty = k_full + ST;
  uint64_t* v_full = k_empty + ST;
  uint64_t* v_empty = v_full + ST;
  uint64_t* s_full = v_empty + ST;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* o_full = p_full + 1;
  uint64_t* drain = o_full + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (p.S + kTile - 1) / kTile;
  const int qt = nq - 1 - (int)blockIdx.x;  // heaviest causal tiles first
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hk = h / (p.Hq / p.Hk);
  const int n_kv = p.causal ? qt + 1 : nq;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_tmem, 4);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, T::kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, L::kQ);
      for (int c = 0; c < NCH; ++c) tma_load_3d(sQ + c * kChunkBytes, &tmQ, q_full, h * HD + c * 64, qt * kTile, b);
      int armed = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % ST;
        const uint32_t ph = (uint32_t)((j / ST) & 1);
        if (!mbar_wait(&k_empty[st], ph ^ 1u, abort_flag, p.status, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&k_full[st], L::kKV);
        for (int c = 0; c < NCH; ++c)
          tma_load_3d(sK + st * L::kKV + c * kChunkBytes, &tmK, &k_full[st], hk * HD + c * 64, j * kTile, b);
        if (!mbar_wait(&v_empty[st], ph ^ 1u, abort_flag, p.status, kErrWaitEmpty)) {
          armed = j;  // K_j in flight but V_j not issued: drain K_j below
          volatile int no_abort = 0;
          mbar_wait(&k_full[st], ph, &no_abort, p.status, kErrWaitFull);
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], L::kKV);
        for (int c = 0; c < NCH; ++c)
          tma_load_3d(sV + st * L::kKV + c * kChunkBytes, &tmV, &v_full[st], hk * HD + c * 64, j * kTile, b);
        armed = j + 1;
      }
      // drain outstanding bulk copies before the CTA can exit
      volatile int no_abort = 0;
      mbar_wait(q_full, 0, &no_abort, p.status, kErrWaitFull);
      for (int j = armed - 1; j >= 0 && j >= armed - ST; --j) {
        mbar_wait(&k_full[j % ST], (uint32_t)((j / ST) & 1), &no_abort, p.status, kErrWaitFull);
        mbar_wait(&v_full[j % ST], (uint32_t)((j / ST) & 1), &no_abort, p.status, kErrWaitFull);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idS = idesc_bf16_f32(128, 128, false, false);
      const uint32_t idPV = idesc_bf16_f32(128, HD, false, true);
      const uint64_t k_desc0 = desc_sw128(smem_u32(sK), 16, 1024);        // K-major K_j
      const uint64_t v_desc0 = desc_sw128(smem_u32(sV), kChunkBytes, 1024);  // MN-major V_j
      const uint32_t q_tm = tbase + T::kQ, p_tm = tbase + T::kP, o_tm = tbase + T::kO;
      bool ok = mbar_wait(q_tmem, 0, abort_flag, p.status, kErrWaitFull);
      tc_fence_after();
      auto issue_s = [&](int j) -> bool {
        const int st = j % ST;
        if (!mbar_wait(&k_full[st], (uint32_t)((j / ST) & 1), abort_flag, p.status, kErrWaitFull)) return false;
        tc_fence_after();
        const uint32_t d = tbase + T::kS + (uint32_t)((j & 1) * 128);
        const uint64_t kd = desc_add(k_desc0, (uint32_t)(st * L::kKV));
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_bf16_ts(d, q_tm + kk * 8, desc_add(kd, (kk >> 2) * kChunkBytes + (kk & 3) * 32), idS, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[j & 1]);
        umma_commit(&k_empty[st]);
        return true;
      };
      for (int j = 0; ok && j < n_kv && j < 2; ++j) ok = issue_s(j);
      for (int j = 0; ok && j < n_kv; ++j) {
        const int buf = j & 1;
        const int st = j % ST;
        if (!mbar_wait(p_full, (uint32_t)(j & 1), abort_flag, p.status, kErrWaitAccum)) break;
        if (!mbar_wait(&v_full[st], (uint32_t)((j / ST) & 1), abort_flag, p.status, kErrWaitFull)) break;
        tc_fence_after();
        const uint64_t vd = desc_add(v_desc0, (uint32_t)(st * L::kKV));
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          umma_bf16_ts(o_tm, p_tm + kk * 8, desc_add(vd, kk * 2048), idPV, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(o_full);
        umma_commit(&v_empty[st]);
        if (j + 2 < n_kv) {
          if (!mbar_wait(&s_empty[buf], (uint32_t)((j >> 1) & 1), abort_flag, p.status, kErrWaitAccEmpty)) break;
          ok = issue_s(j + 2);
        }
      }
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, p.status, kErrWaitAccum);
    }
    __syncwarp();
  } else {
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const int qrow = qt * kTile + r;
    const float sc = p.scale_log2;
    bool ok = wait_lane0(q_full, 0, abort_flag, p.status, kErrWaitFull);
    if (ok) {
      // this thread's query row: swizzled smem -> TMEM lane r (A operand of S = Q K^T)
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const uint8_t* row = sQ + c * kChunkBytes + r * 128;
        uint32_t w[32];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint4 x = *reinterpret_cast<const uint4*>(row + ((u ^ (r & 7)) << 4));
          w[4 * u] = x.x;
          w[4 * u + 1] = x.y;
          w[4 * u + 2] = x.z;
          w[4 * u + 3] = x.w;
        }
        tmem_st_32x32b_x16_nowait(tbase + lane_base + T::kQ + c * 32, w);
        tmem_st_32x32b_x16_nowait(tbase + lane_base + T::kQ + c * 32 + 16, w + 16);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_tmem);
    }
    float m_ref = -INFINITY, l = 0.f;
    for (int j = 0; ok && j < n_kv; ++j) {
      const int buf = j & 1;
      if (!wait_lane0(&s_full[buf], (uint32_t)((j >> 1) & 1), abort_flag, p.status, kErrWaitAccum)) {
        ok = false;
        break;
      }
      ATTN_TRACE_T(64, blockIdx.x, j, 0);
      tc_fence_after();
      float v[128];
      tmem_ld_32x32b_x128(tbase + lane_base + T::kS + (uint32_t)(buf * 128), v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[buf]);
      ATTN_TRACE_T(64, blockIdx.x, j, 1);
      const bool need_mask = (p.causal && j == qt) || (j * kTile + kTile > p.S);
      if (need_mask) {  // keys outside [0, lim) -> -inf (2^-inf = 0 below)
        const int lim = max(0, min(kTile, min(p.causal ? qrow - j * kTile + 1 : kTile, p.S - j * kTile)));
#pragma unroll
        for (int i = 0; i < 128; ++i) v[i] = i < lim ? v[i] : -INFINITY;
      }
      const float mx = max128(v) * sc;
      // a new reference maximum only when the row's scores grew by more than 2^8
      const bool grow = mx > m_ref + kRescaleLog2;
      const float m_new = grow ? mx : m_ref;
      const float alpha = (m_ref == -INFINITY) ? 0.f : ex2_approx(m_ref - m_new);
      ATTN_TRACE_T(64, blockIdx.x, j, 2);
      if (j > 0) {
        // P_{j-1} V_{j-1} must be done: it reads the P buffer and adds into O
        if (!wait_lane0(o_full, (uint32_t)((j - 1) & 1), abort_flag, p.status, kErrWaitAccum)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            float o[32];
            tmem_ld_32x32b_x32(tbase + lane_base + T::kO + c * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st_32x32b_x32(tbase + lane_base + T::kO + c * 32, o);
          }
        }
      }
      ATTN_TRACE_T(64, blockIdx.x, j, 3);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t packed[16];
        if (need_mask)
          fwd_exp32<0>(v + c * 32, sc, -m_use, packed, rs4);
        else
          fwd_exp32<KP>(v + c * 32, sc, -m_use, packed, rs4);
        tmem_st_32x32b_x16_nowait(tbase + lane_base + T::kP + c * 16, packed);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      ATTN_TRACE_T(64, blockIdx.x, j, 4);
      l = l * (grow ? alpha : 1.f) + ((rs4[0] + rs4[1]) + (rs4[2] + rs4[3]));
      m_ref = m_new;
    }
    if (ok && n_kv > 0 &&
        wait_lane0(o_full, (uint32_t)((n_kv - 1) & 1), abort_flag, p.status, kErrWaitAccum)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.o + ((long)b * p.S + qrow) * p.ld_o + (long)h * HD;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        float o[32];
        tmem_ld_32x32b_x32(tbase + lane_base + T::kO + c * 32, o);
        if (qrow < p.S && l > 0.f) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 w = make_uint4(pack_bf16x2(o[8 * u] * inv, o[8 * u + 1] * inv),
                                 pack_bf16x2(o[8 * u + 2] * inv, o[8 * u + 3] * inv),
                                 pack_bf16x2(o[8 * u + 4] * inv, o[8 * u + 5] * inv),
                                 pack_bf16x2(o[8 * u + 6] * inv, o[8 * u + 7] * inv));
            *reinterpret_cast<uint4*>(orow + c * 32 + 8 * u) = w;
          }
        }
      }
      if (qrow < p.S && l > 0.f) p.lse[((long)b * p.Hq + h) * p.S + qrow] = (m_ref + log2f(l)) * kLn2;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, T::kCols);
  }
}

// Two query tiles per CTA (HD 64): softmax warpgroups 0 and 1 own query tiles
// 2c and 2c+1 and share every K_j / V_j load.  While one warpgroup is in its
// exp2 phase (bound by the special-function unit) the other loads S, takes row
// maxima and waits on the tensor core, so the SFU stays busy.  TMEM: S_t
// [t*128, +128), O_t [256 + t*64, +64), P_t [384 + t*64, +64); Q stays in
// shared memory (S = Q K^T reads both operands from there).
struct Fwd2QSmem {
  static constexpr int ST = 4;
  static constexpr int kQ = kChunkBytes;
  static constexpr int kKV = kChunkBytes;
  static constexpr int kBytes = 2 * kQ + 2 * ST * kKV;
};
constexpr int kFwd2QThreads = 320;

template <int KP = kFwdPolyPairs>
__global__ void __launch_bounds__(kFwd2QThreads, 1)
    attn_fwd_2q_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  using L = Fwd2QSmem;
  constexpr int HD = 64, ST = L::ST;
  constexpr uint32_t kCols = 512, cS = 0, cO = 256, cP = 384;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((base_u32 + 1023u) & ~1023u) - base_u32);
  uint8_t* sQ = smem;                // [2] tiles
  uint8_t* sK = sQ + 2 * L::kQ;      // [ST]
  uint8_t* sV = sK + ST * L::kKV;    // [ST]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + ST * L::kKV);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + ST;
  uint64_t* v_full = k_empty + ST;
  uint64_t* v_empty = v_full + ST;
  uint64_t* s_full = v_empty + ST;  // [2] per tile
  uint64_t* s_empty = s_full + 2;   // [2]
  uint64_t* p_full = s_empty + 2;   // [2]
  uint64_t* o_full = p_full + 2;    // [2]
  uint64_t* drain = o_full + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (p.S + kTile - 1) / kTile;
  const int nblk = (nq + 1) / 2;
  const int blk = nblk - 1 - (int)blockIdx.x;  // heaviest causal blocks first
  const int qt0 = 2 * blk;
  const bool has1 = qt0 + 1 < nq;
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hk = h / (p.Hq / p.Hk);
  const int n0 = p.causal ? qt0 + 1 : nq;
  const int n1 = has1 ? (p.causal ? qt0 + 2 : nq) : 0;
  const int n_kv = max(n0, n1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&s_empty[t], 4);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_full[t], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, (has1 ? 2 : 1) * L::kQ);
      tma_load_3d(sQ, &tmQ, q_full, h * HD, qt0 * kTile, b);
      if (has1) tma_load_3d(sQ + L::kQ, &tmQ, q_full, h * HD, (qt0 + 1) * kTile, b);
      int armed = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % ST;
        const uint32_t ph = (uint32_t)((j / ST) & 1);
        if (!mbar_wait(&k_empty[st], ph ^ 1u, abort_flag, p.status, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&k_full[st], L::kKV);
        tma_load_3d(sK + st * L::kKV, &tmK, &k_full[st], hk * HD, j * kTile, b);
        FWD_TRACE(j, 12);
        if (!mbar_wait(&v_empty[st], ph ^ 1u, abort_flag, p.status, kErrWaitEmpty)) {
          armed = j;  // K_j in flight but V_j not issued: drain K_j below
          volatile int no_abort = 0;
          mbar_wait(&k_full[st], ph, &no_abort, p.status, kErrWaitFull);
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], L::kKV);
        tma_load_3d(sV + st * L::kKV, &tmV, &v_full[st], hk * HD, j * kTile, b);
        FWD_TRACE(j, 13);
        armed = j + 1;
      }
      volatile int no_abort = 0;
      mbar_wait(q_full, 0, &no_abort, p.status, kErrWaitFull);
      for (int j = armed - 1; j >= 0 && j >= armed - ST; --j) {
        mbar_wait(&k_full[j % ST], (uint32_t)((j / ST) & 1), &no_abort, p.status, kErrWaitFull);
        mbar_wait(&v_full[j % ST], (uint32_t)((j / ST) & 1), &no_abort, p.status, kErrWaitFull);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idS = idesc_bf16_f32(128, 128, false, false);
      const uint32_t idPV = idesc_bf16_f32(128, HD, false, true);
      const uint64_t q_desc0 = desc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t k_desc0 = desc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t v_desc0 = desc_sw128(smem_u32(sV), kChunkBytes, 1024);
      const int nt[2] = {n0, n1};
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, kErrWaitFull);
      // S_t(j) = Q_t K_j^T (softmax t has loaded S_t(j-1) out of TMEM)
      auto issue_s = [&](int t, int j, uint64_t kd) -> bool {
        if (j > 0 && !mbar_wait(&s_empty[t], (uint32_t)((j - 1) & 1), abort_flag, p.status, kErrWaitAccEmpty))
          return false;
        tc_fence_after();
        const uint64_t qd = desc_add(q_desc0, (uint32_t)(t * L::kQ));
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_bf16_ss(tbase + cS + (uint32_t)(t * 128), desc_add(qd, kk * 32), desc_add(kd, kk * 32), idS,
                       kk > 0 ? 1u : 0u);
        umma_commit(&s_full[t]);
        return true;
      };
      // O_t += P_t(j) V_j (softmax t has written P_t(j) and rescaled O_t)
      auto issue_pv = [&](int t, int j, uint64_t vd) -> bool {
        if (!mbar_wait(&p_full[t], (uint32_t)(j & 1), abort_flag, p.status, kErrWaitAccum)) return false;
        FWD_TRACE(j, 2 + t);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          umma_bf16_ts(tbase + cO + (uint32_t)(t * HD), tbase + cP + (uint32_t)(t * 64 + kk * 8),
                       desc_add(vd, kk * 2048), idPV, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&o_full[t]);
        return true;
      };
      auto issue_pvs = [&](int j) -> bool {
        const int st = j % ST;
        if (!mbar_wait(&v_full[st], (uint32_t)((j / ST) & 1), abort_flag, p.status, kErrWaitFull)) return false;
        const uint64_t vd = desc_add(v_desc0, (uint32_t)(st * L::kKV));
        for (int t = 0; t < 2; ++t)
          if (j < nt[t] && !issue_pv(t, j, vd)) return false;
        umma_commit(&v_empty[st]);
        return true;
      };
      for (int j = 0; ok && j < n_kv; ++j) {
        const int st = j % ST;
        if (!mbar_wait(&k_full[st], (uint32_t)((j / ST) & 1), abort_flag, p.status, kErrWaitFull)) {
          ok = false;
          break;
        }
        const uint64_t kd = desc_add(k_desc0, (uint32_t)(st * L::kKV));
        FWD_TRACE(j, 0);
        for (int t = 0; ok && t < 2; ++t)
          if (j < nt[t]) ok = issue_s(t, j, kd);
        if (!ok) break;
        FWD_TRACE(j, 1);
        umma_commit(&k_empty[st]);
        if (j > 0) ok = issue_pvs(j - 1);
      }
      if (ok && n_kv > 0) issue_pvs(n_kv - 1);
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, p.status, kErrWaitAccum);
    }
    __syncwarp();
  } else {
    const int t = (warp - 2) >> 2;  // query tile of this warpgroup
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const int qt = qt0 + t;
    const int n_t = t == 0 ? n0 : n1;
    const int qrow = qt * kTile + r;
    const float sc = p.scale_log2;
    const uint32_t s_tm = tbase + lane_base + cS + (uint32_t)(t * 128);
    const uint32_t o_tm = tbase + lane_base + cO + (uint32_t)(t * HD);
    const uint32_t p_tm = tbase + lane_base + cP + (uint32_t)(t * 64);
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_t; ++j) {
      if (!wait_lane0(&s_full[t], (uint32_t)(j & 1), abort_flag, p.status, kErrWaitAccum)) {
        ok = false;
        break;
      }
      if (q4 == 0 && lane == 0) FWD_TRACE(j, 4 + 4 * t);
      tc_fence_after();
      float v[128];
      tmem_ld_32x32b_x128(s_tm, v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[t]);
      const bool need_mask = (p.causal && j == qt) || (j * kTile + kTile > p.S);
      if (need_mask) {  // keys outside [0, lim) -> -inf (2^-inf = 0 below)
        const int lim = max(0, min(kTile, min(p.causal ? qrow - j * kTile + 1 : kTile, p.S - j * kTile)));
#pragma unroll
        for (int i = 0; i < 128; ++i) v[i] = i < lim ? v[i] : -INFINITY;
      }
      const float mx = max128(v) * sc;
      const bool grow = mx > m_ref + kRescaleLog2;
      const float m_new = grow ? mx : m_ref;
      const float alpha = (m_ref == -INFINITY) ? 0.f : ex2_approx(m_ref - m_new);
      if (q4 == 0 && lane == 0) FWD_TRACE(j, 5 + 4 * t);
      if (j > 0) {
        // P_t(j-1) V_{j-1} must be done: it reads P_t and adds into O_t
        if (!wait_lane0(&o_full[t], (uint32_t)((j - 1) & 1), abort_flag, p.status, kErrWaitAccum)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            float o[32];
            tmem_ld_32x32b_x32(o_tm + c * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st_32x32b_x32(o_tm + c * 32, o);
          }
        }
      }
      if (q4 == 0 && lane == 0) FWD_TRACE(j, 6 + 4 * t);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t packed[16];
        if (need_mask)
          fwd_exp32<0>(v + c * 32, sc, -m_use, packed, rs4);
        else
          fwd_exp32<KP>(v + c * 32, sc, -m_use, packed, rs4);
        tmem_st_32x32b_x16_nowait(p_tm + c * 16, packed);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
      if (q4 == 0 && lane == 0) FWD_TRACE(j, 7 + 4 * t);
      l = l * (grow ? alpha : 1.f) + ((rs4[0] + rs4[1]) + (rs4[2] + rs4[3]));
      m_ref = m_new;
    }
    if (ok && n_t > 0 && wait_lane0(&o_full[t], (uint32_t)((n_t - 1) & 1), abort_flag, p.status, kErrWaitAccum)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.o + ((long)b * p.S + qrow) * p.ld_o + (long)h * HD;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        float o[32];
        tmem_ld_32x32b_x32(o_tm + c * 32, o);
        if (qrow < p.S && l > 0.f) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 w = make_uint4(pack_bf16x2(o[8 * u] * inv, o[8 * u + 1] * inv),
                                 pack_bf16x2(o[8 * u + 2] * inv, o[8 * u + 3] * inv),
                                 pack_bf16x2(o[8 * u + 4] * inv, o[8 * u + 5] * inv),
                                 pack_bf16x2(o[8 * u + 6] * inv, o[8 * u + 7] * inv));
            *reinterpret_cast<uint4*>(orow + c * 32 + 8 * u) = w;
          }
        }
      }
      if (qrow < p.S && l > 0.f) p.lse[((long)b * p.Hq + h) * p.S + qrow] = (m_ref + log2f(l)) * kLn2;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kCols);
  }
}

// Two 32-column TMEM loads in flight, then one wait.
__device__ __forceinline__ void tmem_ld2_x32(uint32_t ta, float* a, uint32_t tb, float* b) {
  if (!MT_CHECK((ta & 0xFFFFu) + 32u <= 512u && (tb & 0xFFFFu) + 32u <= 512u, kErrCheckTmem)) return;
  uint32_t r[32], q[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3]), "=r"(q[4]), "=r"(q[5]), "=r"(q[6]), "=r"(q[7]),
        "=r"(q[8]), "=r"(q[9]), "=r"(q[10]), "=r"(q[11]), "=r"(q[12]), "=r"(q[13]), "=r"(q[14]), "=r"(q[15]),
        "=r"(q[16]), "=r"(q[17]), "=r"(q[18]), "=r"(q[19]), "=r"(q[20]), "=r"(q[21]), "=r"(q[22]), "=r"(q[23]),
        "=r"(q[24]), "=r"(q[25]), "=r"(q[26]), "=r"(q[27]), "=r"(q[28]), "=r"(q[29]), "=r"(q[30]), "=r"(q[31])
      : "r"(ta), "r"(tb)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    a[i] = __uint_as_float(r[i]);
    b[i] = __uint_as_float(q[i]);
  }
}

// ------------------------------------------------------------------ forward, ping-pong
// Two query tiles per CTA (both head dims).  Softmax warpgroup t owns query
// tile t; the single MMA thread issues, per KV tile j,
//     PV_0(j), S_0(j+1), PV_1(j), S_1(j+1)
// so while one warpgroup runs its exponentials the tensor core computes the
// other tile's products, and the two warpgroups settle half a step apart.
// TMEM: S_t at columns [128 t, +128); P_t (bf16 pairs) overwrites the first 64
// columns of S_t once they are read; O_t at [256 + 128 t, +HD).  The MMAs of a
// CTA run in issue order, so S_t(j+1) overwrites P_t(j) only after PV_t(j) has
// read it, and s_full_t(j) (committed after S_t(j), itself issued after
// PV_t(j-1)) also tells the softmax that O_t may be rescaled.  Q_t, K_j and V_j
// are shared-memory operands (SW128 64-column chunks).
template <int HD>
struct FwdPPSmem {
  static constexpr int ST = HD == 64 ? 4 : 2;  // K/V stages
  static constexpr int kTileB = HD / 64 * kChunkBytes;
  static constexpr int kBytes = 2 * kTileB + 2 * ST * kTileB;
};
constexpr int kFwdPPThreads = 320;

template <int HD, int KP>
__global__ void __launch_bounds__(kFwdPPThreads, 1)
    attn_fwd_pp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  using L = FwdPPSmem<HD>;
  constexpr int ST = L::ST, NCH = HD / 64;
  constexpr uint32_t kCols = 512, cS = 0, cO = 256;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((base_u32 + 1023u) & ~1023u) - base_u32);
  uint8_t* sQ = smem;                 // [2] tiles
  uint8_t* sK = sQ + 2 * L::kTileB;   // [ST]
  uint8_t* sV = sK + ST * L::kTileB;  // [ST]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + ST * L::kTileB);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + ST;
  uint64_t* v_full = k_empty + ST;
  uint64_t* v_empty = v_full + ST;
  uint64_t* s_full = v_empty + ST;  // [2]
  uint64_t* p_full = s_full + 2;    // [2]
  uint64_t* o_full = p_full + 2;    // [2]
  uint64_t* tok = o_full + 2;       // [2]: tok[t] = the other warpgroup finished an exponential phase
  uint64_t* drain = tok + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (p.S + kTile - 1) / kTile;
  const int nblk = (nq + 1) / 2;
  const int blk = nblk - 1 - (int)blockIdx.x;  // heaviest causal blocks first
  const int qt0 = 2 * blk;
  const bool has1 = qt0 + 1 < nq;
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hk = h / (p.Hq / p.Hk);
  const int n0 = p.causal ? qt0 + 1 : nq;
  const int n1 = has1 ? (p.causal ? qt0 + 2 : nq) : 0;
  const int n_kv = max(n0, n1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_full[t], 1);
      mbar_init(&tok[t], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, (has1 ? 2 : 1) * L::kTileB);
      for (int t = 0; t < (has1 ? 2 : 1); ++t)
        for (int c = 0; c < NCH; ++c)
          tma_load_3d(sQ + t * L::kTileB + c * kChunkBytes, &tmQ, q_full, h * HD + c * 64, (qt0 + t) * kTile, b);
      int armed = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % ST;
        const uint32_t ph = (uint32_t)((j / ST) & 1);
        if (!mbar_wait(&k_empty[st], ph ^ 1u, abort_flag, p.status, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&k_full[st], L::kTileB);
        for (int c = 0; c < NCH; ++c)
          tma_load_3d(sK + st * L::kTileB + c * kChunkBytes, &tmK, &k_full[st], hk * HD + c * 64, j * kTile, b);
        if (!mbar_wait(&v_empty[st], ph ^ 1u, abort_flag, p.status, kErrWaitEmpty)) {
          armed = j;  // K_j in flight but V_j not issued: drain K_j below
          volatile int no_abort = 0;
          mbar_wait(&k_full[st], ph, &no_abort, p.status, kErrWaitFull);
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], L::kTileB);
        for (int c = 0; c < NCH; ++c)
          tma_load_3d(sV + st * L::kTileB + c * kChunkBytes, &tmV, &v_full[st], hk * HD + c * 64, j * kTile, b);
        armed = j + 1;
      }
      // drain outstanding bulk copies before the CTA can exit
      volatile int no_abort = 0;
      mbar_wait(q_full, 0, &no_abort, p.status, kErrWaitFull);
      for (int j = armed - 1; j >= 0 && j >= armed - ST; --j) {
        mbar_wait(&k_full[j % ST], (uint32_t)((j / ST) & 1), &no_abort, p.status, kErrWaitFull);
        mbar_wait(&v_full[j % ST], (uint32_t)((j / ST) & 1), &no_abort, p.status, kErrWaitFull);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idS = idesc_bf16_f32(128, 128, false, false);
      const uint32_t idPV = idesc_bf16_f32(128, HD, false, true);
      const uint64_t q_desc0 = desc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t k_desc0 = desc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t v_desc0 = desc_sw128(smem_u32(sV), kChunkBytes, 1024);
      const int nt[2] = {n0, n1};
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, kErrWaitFull);
      tc_fence_after();
      // S_t(j) = Q_t K_j^T into S_t
      auto issue_s = [&](int t, int j) {
        const uint64_t qd = desc_add(q_desc0, (uint32_t)(t * L::kTileB));
        const uint64_t kd = desc_add(k_desc0, (uint32_t)((j % ST) * L::kTileB));
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * kChunkBytes + (kk & 3) * 32);
          umma_bf16_ss(tbase + cS + (uint32_t)(t * 128), desc_add(qd, off), desc_add(kd, off), idS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      if (ok && n_kv > 0) {
        ok = mbar_wait(&k_full[0], 0, abort_flag, p.status, kErrWaitFull);
        if (ok) {
          tc_fence_after();
          for (int t = 0; t < 2; ++t)
            if (nt[t] > 0) issue_s(t, 0);
          umma_commit(&k_empty[0]);
        }
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int st = j % ST;
        if (!mbar_wait(&v_full[st], (uint32_t)((j / ST) & 1), abort_flag, p.status, kErrWaitFull)) break;
        const uint64_t vd = desc_add(v_desc0, (uint32_t)(st * L::kTileB));
        bool k_next = false;  // K_{j+1} resident
        for (int t = 0; ok && t < 2; ++t) {
          if (j >= nt[t]) continue;
          // O_t += P_t(j) V_j once softmax t has written P_t(j) (and rescaled O_t)
          if (!mbar_wait(&p_full[t], (uint32_t)(j & 1), abort_flag, p.status, kErrWaitAccum)) {
            ok = false;
            break;
          }
          FWD_TRACE(j, 2 + t);
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kTile / 16; ++kk)
            umma_bf16_ts(tbase + cO + (uint32_t)(t * 128), tbase + cS + (uint32_t)(t * 128 + kk * 8),
                         desc_add(vd, kk * 2048), idPV, (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&o_full[t]);
          if (j + 1 < nt[t]) {
            if (!k_next) {
              const int s1 = (j + 1) % ST;
              if (!mbar_wait(&k_full[s1], (uint32_t)(((j + 1) / ST) & 1), abort_flag, p.status, kErrWaitFull)) {
                ok = false;
                break;
              }
              tc_fence_after();
              k_next = true;
            }
            issue_s(t, j + 1);
          }
        }
        if (!ok) break;
        umma_commit(&v_empty[st]);
        if (k_next) umma_commit(&k_empty[(j + 1) % ST]);
      }
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, p.status, kErrWaitAccum);
    }
    __syncwarp();
  } else {
    const int t = (warp - 2) >> 2;  // query tile of this warpgroup
    const int q4 = warp & 3;        // TMEM lane quarter of this warp
    const int r = q4 * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const int qt = qt0 + t;
    const int n_t = t == 0 ? n0 : n1;
    const int qrow = qt * kTile + r;
    const float sc = p.scale_log2;
    const uint32_t s_tm = tbase + lane_base + cS + (uint32_t)(t * 128);
    const uint32_t o_tm = tbase + lane_base + cO + (uint32_t)(t * 128);
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_t; ++j) {
      if (!wait_lane0(&s_full[t], (uint32_t)(j & 1), abort_flag, p.status, kErrWaitAccum)) {
        ok = false;
        break;
      }
      if (q4 == 0 && lane == 0) FWD_TRACE(j, 4 + 4 * t);
      tc_fence_after();
      const bool need_mask = (p.causal && j == qt) || (j * kTile + kTile > p.S);
      // keys at or past lim are masked (-inf; 2^-inf = 0 on the special-function path)
      const int lim = need_mask ? max(0, min(kTile, min(p.causal ? qrow - j * kTile + 1 : kTile, p.S - j * kTile)))
                                : kTile;
      // pass 1: row maximum of S_t(j)
      float mx = -INFINITY;
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        float a[32], e[32];
        tmem_ld2_x32(s_tm + (uint32_t)(64 * c2), a, s_tm + (uint32_t)(64 * c2 + 32), e);
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            a[i] = 64 * c2 + i < lim ? a[i] : -INFINITY;
            e[i] = 64 * c2 + 32 + i < lim ? e[i] : -INFINITY;
          }
        }
        mx = max32(e, max32(a, mx));
      }
      mx *= sc;
      // a new reference maximum only when the row's scores grew by more than 2^8
      const bool grow = mx > m_ref + kRescaleLog2;
      const float m_new = grow ? mx : m_ref;
      const float alpha = (m_ref == -INFINITY) ? 0.f : ex2_approx(m_ref - m_new);
      if (q4 == 0 && lane == 0) FWD_TRACE(j, 5 + 4 * t);
      if (j > 0 && __any_sync(0xffffffffu, grow)) {  // PV_t(j-1) is complete: S_t(j) was issued after it
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          float o[32];
          tmem_ld_32x32b_x32(o_tm + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st_32x32b_x32(o_tm + c * 32, o);
        }
      }
      if (q4 == 0 && lane == 0) FWD_TRACE(j, 6 + 4 * t);
      // With p.alternate the exponential phases of the two warpgroups take turns
      // (tile 0 step j, tile 1 step j, tile 0 step j+1, ...) so the special-function
      // and FMA pipes serve one warpgroup at a time while the tensor core works
      // for the other.  The turn is an mbarrier (bounded wait), not a named barrier.
      if (p.alternate) {
        const bool wait_turn = t == 0 ? (has1 && j >= 1) : (j < n0);
        if (wait_turn &&
            !wait_lane0(&tok[t], (uint32_t)((t == 0 ? j - 1 : j) & 1), abort_flag, p.status, kErrWaitAccum)) {
          ok = false;
          break;
        }
      }
      // pass 2: P = 2^(s sc - m) as bf16 over the columns of S already read
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        uint32_t packed[16];
        tmem_ld_32x32b_x32(s_tm + (uint32_t)(32 * c), v);
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 32 * c + i < lim ? v[i] : -INFINITY;
          fwd_exp32<0>(v, sc, -m_use, packed, rs4);
        } else {
          fwd_exp32<KP>(v, sc, -m_use, packed, rs4);
        }
        tmem_st_32x32b_x16_nowait(s_tm + (uint32_t)(16 * c), packed);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
      if (p.alternate && lane == 0) {
        // tile 1 waits for every step of tile 0; tile 0 (from step 1) for tile 1's steps 0 .. n0-2
        if (t == 0 ? has1 : (j + 1 < n0)) mbar_arrive(&tok[1 - t]);
      }
      if (q4 == 0 && lane == 0) FWD_TRACE(j, 7 + 4 * t);
      l = l * (grow ? alpha : 1.f) + ((rs4[0] + rs4[1]) + (rs4[2] + rs4[3]));
      m_ref = m_new;
    }
    if (ok && n_t > 0 && wait_lane0(&o_full[t], (uint32_t)((n_t - 1) & 1), abort_flag, p.status, kErrWaitAccum)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.o + ((long)b * p.S + qrow) * p.ld_o + (long)h * HD;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        float o[32];
        tmem_ld_32x32b_x32(o_tm + c * 32, o);
        if (qrow < p.S && l > 0.f) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 w = make_uint4(pack_bf16x2(o[8 * u] * inv, o[8 * u + 1] * inv),
                                 pack_bf16x2(o[8 * u + 2] * inv, o[8 * u + 3] * inv),
                                 pack_bf16x2(o[8 * u + 4] * inv, o[8 * u + 5] * inv),
                                 pack_bf16x2(o[8 * u + 6] * inv, o[8 * u + 7] * inv));
            *reinterpret_cast<uint4*>(orow + c * 32 + 8 * u) = w;
          }
        }
      }
      if (qrow < p.S && l > 0.f) p.lse[((long)b * p.Hq + h) * p.S + qrow] = (m_ref + log2f(l)) * kLn2;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kCols);
  }
}

// ------------------------------------------------------------------ backward

struct BwdParams {
  const float* lse;
  const float* delta;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  long ld_dk, ld_dv;
  int B, S, Hq, Hk;
  float scale_log2, scale;
  int causal;
  uint32_t* status;
};

template <int HD>
struct BwdSmem {
  // K/V stages: HD=64 double-buffers them so the next work item's K/V arrive while this one runs
  static constexpr int KVST = HD == 64 ? 2 : 1;
  // Q/dO stages: loads run two tiles ahead for HD=64 (their latency exceeds a tile's work)
  static constexpr int STQ = HD == 64 ? 3 : 1;
  static constexpr int kT = HD / 64 * kChunkBytes;   // one [128 x HD] bf16 tile
  static constexpr int kPT = 2 * kChunkBytes;        // [128 x 128] bf16
  static constexpr int kDQ = kTile * 128;            // [128 rows x 32 fp32] staging chunk (SW128)
  static constexpr int NDQ = HD == 64 ? 1 : 2;       // staging chunks; dQ drains in HD/32/NDQ rounds
  static constexpr int NDQB = 1;                     // dQ accumulators in TMEM
  // HD=64: P^T lives in TMEM (A operand of dV += P^T dO), so only dS^T is staged in smem
  static constexpr bool kPtTmem = HD == 64;
  static constexpr int kBytes = 2 * KVST * kT + 2 * STQ * kT + (kPtTmem ? 1 : 2) * kPT + NDQ * kDQ +
                                2 * STQ * kTile * 4;
};

// Work items of the persistent backward: (kv tile, batch, kv head), heaviest
// first (a causal kv tile kt meets nq - kt query tiles).  CTA c takes item c in
// round 0, item 2C-1-c in round 1, 2C+c in round 2, ...: alternating direction
// pairs heavy with light items, so the CTAs finish close together.
struct BwdItem {
  int kt, b, hk, qt0, per_head, n_it;
};

__device__ __forceinline__ int bwd_item_index(int round, int ctas) {
  const int base = round * ctas;
  return (round & 1) ? base + ctas - 1 - (int)blockIdx.x : base + (int)blockIdx.x;
}

__device__ __forceinline__ BwdItem bwd_item(int idx, int nq, int B, int Hk, int G, int causal) {
  BwdItem w;
  const int bh = idx % (B * Hk);
  w.kt = idx / (B * Hk);
  w.b = bh / Hk;
  w.hk = bh % Hk;
  w.qt0 = causal ? w.kt : 0;
  w.per_head = nq - w.qt0;
  w.n_it = G * w.per_head;
  return w;
}

// TMA warp, MMA warp, two softmax warpgroups (query columns 0-63 / 64-127), dQ warpgroup
constexpr int kBwdThreads = 448;
constexpr int kBwdSoftmaxWarps = 8;


// Row `row` (32 fp32 = 128 bytes) of a [128 x 32] fp32 tile in the SW128 layout the TMA expects.
__device__ __forceinline__ void store_row_f32_sw128(uint8_t* tile, int row, const float* v) {
  uint8_t* line = tile + row * 128;
#pragma unroll
  for (int u = 0; u < 8; ++u)
    *reinterpret_cast<float4*>(line + ((u ^ (row & 7)) << 4)) =
        make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
}

// Bulk tensor reduce-add of a shared-memory tile into global memory.
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  // fp32 map: x 16-byte aligned; a reduce may not start at a negative coordinate
  if (!MT_CHECK((x & 3) == 0 && x >= 0 && y >= 0 && z >= 0, kErrCheckTma)) return;
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Share of the backward's exponentials on the FMA pipe (pairs of 16); masked
// tiles use the special-function unit only (exact zeros).
#ifndef MT_BWD_POLY_PAIRS
#define MT_BWD_POLY_PAIRS 5
#endif
constexpr int kBwdPolyPairs = MT_BWD_POLY_PAIRS;

// P^T / dS^T for 32 query columns of one key row.  MASK: causal diagonal tile
// or key rows past S; otherwise every entry is live.  Queries past S carry
// lse = +inf, so their P is 0 on either path.
template <bool MASK, int KP>
__device__ __forceinline__ void bwd_softmax32(const float* sv, const float* dp, const float* lse2, const float* dlt,
                                              float sc, int q0, int krow, bool key_dead, uint32_t* pk,
                                              uint32_t* dk) {
  // Pairs of columns go through the packed f32x2 pipe; bf16 packing is integer
  // arithmetic, so the special-function pipe only runs the exponentials.
  const float4* L4 = reinterpret_cast<const float4*>(lse2);
  const float4* D4 = reinterpret_cast<const float4*>(dlt);
  const uint64_t sc2 = f2pack(sc, sc);
#pragma unroll
  for (int j4 = 0; j4 < 8; ++j4) {
    const float4 l = L4[j4], d = D4[j4];
    const uint64_t neg_l[2] = {f2pack(-l.x, -l.y), f2pack(-l.z, -l.w)};
    const uint64_t dv[2] = {f2pack(d.x, d.y), f2pack(d.z, d.w)};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = 4 * j4 + 2 * h;
      const uint64_t x = fma_f32x2(f2pack(sv[j], sv[j + 1]), sc2, neg_l[h]);
      float e0, e1;
      uint64_t e2;
      if (!MASK && KP > 0 && poly_pair<KP>(2 * j4 + h)) {
        e2 = ex2_poly_x2(x);
        f2unpack(e2, e0, e1);
      } else {
        float a0, a1;
        f2unpack(x, a0, a1);
        e0 = ex2_approx(a0);
        e1 = ex2_approx(a1);
        if (MASK) {
          if (key_dead || q0 + j < krow) e0 = 0.f;
          if (key_dead || q0 + j + 1 < krow) e1 = 0.f;
        }
        e2 = f2pack(e0, e1);
      }
      float ds0, ds1;
      f2unpack(mul_f32x2(e2, sub_f32x2(f2pack(dp[j], dp[j + 1]), dv[h])), ds0, ds1);
      pk[2 * j4 + h] = pack_bf16x2_int(e0, e1);
      dk[2 * j4 + h] = pack_bf16x2_int(ds0, ds1);
    }
  }
}

template <int HD, int KP = kBwdPolyPairs>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmDQ, const BwdParams p) {
  using L = BwdSmem<HD>;
  constexpr int STQ = L::STQ;
  constexpr int KVST = L::KVST;
  constexpr int NCH = HD / 64;
  constexpr uint32_t TMEM_COLS = 512;
  constexpr int NDQB = L::NDQB;
  // TMEM columns: S^T [0,128), dP^T [128,256), dV [256,256+HD), dK [256+HD, 256+2HD);
  // HD=64: dQ [384,448) and bf16 P^T [448,512); HD=128: dQ aliased onto S^T, P^T in smem.
  constexpr uint32_t cS = 0, cDP = 128, cDV = 256, cDK = 256 + HD, cDQ = (HD == 64) ? 384 : 0, cPT = 448;
  constexpr bool PT_TMEM = L::kPtTmem;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((base_u32 + 1023u) & ~1023u) - base_u32);
  uint8_t* sK = smem;                      // [KVST]
  uint8_t* sV = sK + KVST * L::kT;         // [KVST]
  uint8_t* sQ = sV + KVST * L::kT;         // [STQ]
  uint8_t* sDO = sQ + STQ * L::kT;         // [STQ]
  uint8_t* sPT = sDO + STQ * L::kT;        // unused when P^T lives in TMEM
  uint8_t* sDST = sPT + (PT_TMEM ? 0 : L::kPT);
  uint8_t* sDQ = sDST + L::kPT;                                   // NDQ x [128 x 32] fp32
  float* sLse = reinterpret_cast<float*>(sDQ + L::NDQ * L::kDQ);  // [STQ][128]
  float* sDelta = sLse + STQ * kTile;                              // [STQ][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDelta + STQ * kTile);
  uint64_t* kv_full = bars;                // [KVST]
  uint64_t* kv_empty = kv_full + KVST;     // [KVST] every MMA of the item that read this K/V stage is done
  uint64_t* qdo_full = kv_empty + KVST;
  uint64_t* qdo_empty = qdo_full + STQ;
  uint64_t* s_full = qdo_empty + STQ;
  uint64_t* ds_full = s_full + 1;
  uint64_t* ds_empty = ds_full + 1;
  uint64_t* dq_full = ds_empty + 1;     // [NDQB]
  uint64_t* s_empty = dq_full + NDQB;   // S^T / dP^T TMEM may be overwritten
  uint64_t* dq_empty = s_empty + 1;     // [NDQB] dQ TMEM may be overwritten
  uint64_t* dkv_full = dq_empty + NDQB;  // the item's dK / dV are complete in TMEM
  uint64_t* dkv_empty = dkv_full + 1;    // the epilogue has read them out
  uint32_t* tslot = reinterpret_cast<uint32_t*>(dkv_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (p.S + kTile - 1) / kTile;
  const int G = p.Hq / p.Hk;
  const int n_items = nq * p.B * p.Hk;
  const int ctas = (int)gridDim.x;
  const int rounds = (n_items + ctas - 1) / ctas;
  // every role walks this CTA's items in the same order:
  //   for (r < rounds) { idx = bwd_item_index(r, ctas); if (idx >= n_items) continue; ... }

  if (threadIdx.x == 0) {
    for (int s = 0; s < KVST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < STQ; ++s) {
      mbar_init(&qdo_full[s], 2);  // the Q / dO copies, and the lse / delta rows
      mbar_init(&qdo_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(ds_full, kBwdSoftmaxWarps);
    mbar_init(ds_empty, 1);
    for (int j = 0; j < NDQB; ++j) {
      mbar_init(&dq_full[j], 1);
      mbar_init(&dq_empty[j], 4);
    }
    mbar_init(s_empty, HD == 64 ? kBwdSoftmaxWarps : 4);
    mbar_init(dkv_full, 1);
    mbar_init(dkv_empty, 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp == 0) {
    // ---------------- TMA warp: K/V per item, Q/dO (+ lse, delta rows) per query tile
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmDO);
      tma_prefetch_desc(&tmDQ);
    }
    int ni = 0, gq = 0;          // items and query tiles issued so far
    bool ok = true;
    for (int r = 0; ok && r < rounds; ++r) {
      const int idx = bwd_item_index(r, ctas);
      if (idx >= n_items) continue;
      const BwdItem w = bwd_item(idx, nq, p.B, p.Hk, G, p.causal);
      const int ks = ni % KVST;
      if (!wait_lane0(&kv_empty[ks], (uint32_t)((ni / KVST) & 1) ^ 1u, abort_flag, p.status, kErrWaitEmpty)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&kv_full[ks], 2 * L::kT);
        for (int c = 0; c < NCH; ++c) {
          tma_load_3d(sK + ks * L::kT + c * kChunkBytes, &tmK, &kv_full[ks], w.hk * HD + c * 64, w.kt * kTile, w.b);
          tma_load_3d(sV + ks * L::kT + c * kChunkBytes, &tmV, &kv_full[ks], w.hk * HD + c * 64, w.kt * kTile, w.b);
        }
      }
      ++ni;
      for (int it = 0; it < w.n_it; ++it, ++gq) {
        const int h = w.hk * G + it / w.per_head;
        const int qt = w.qt0 + it % w.per_head;
        const int st = gq % STQ;
        if (!wait_lane0(&qdo_empty[st], (uint32_t)((gq / STQ) & 1) ^ 1u, abort_flag, p.status, kErrWaitEmpty)) {
          ok = false;
          break;
        }
        if (lane == 0) BWD_TRACE(gq, 10);
        // the bulk copies first, then the lse / delta rows while they fly: the stage is
        // full once both have arrived (two arrivals on qdo_full)
        if (lane == 0) {
          mbar_arrive_expect_tx(&qdo_full[st], 2 * L::kT);
          for (int c = 0; c < NCH; ++c) {
            tma_load_3d(sQ + st * L::kT + c * kChunkBytes, &tmQ, &qdo_full[st], h * HD + c * 64, qt * kTile, w.b);
            tma_load_3d(sDO + st * L::kT + c * kChunkBytes, &tmDO, &qdo_full[st], h * HD + c * 64, qt * kTile, w.b);
          }
        }
        const long row0 = ((long)w.b * p.Hq + h) * p.S;
        for (int i = lane; i < kTile; i += 32) {
          const int q = qt * kTile + i;
          sLse[st * kTile + i] = q < p.S ? p.lse[row0 + q] * kLog2e : INFINITY;
          sDelta[st * kTile + i] = q < p.S ? p.delta[row0 + q] : 0.f;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&qdo_full[st]);
      }
    }
    if (lane == 0) {  // every bulk copy issued has landed before the CTA can retire
      volatile int no_abort = 0;
      for (int n = ni - 1; n >= 0 && n >= ni - KVST; --n)
        mbar_wait(&kv_full[n % KVST], (uint32_t)((n / KVST) & 1), &no_abort, p.status, kErrWaitFull);
      for (int g = gq - 1; g >= 0 && g >= gq - STQ; --g)
        mbar_wait(&qdo_full[g % STQ], (uint32_t)((g / STQ) & 1), &no_abort, p.status, kErrWaitFull);
    }
  } else if (warp == 1) {
    // ---------------- MMA warp: one elected thread issues every tcgen05.mma
    if (elect_one()) {
      const uint32_t idSS = idesc_bf16_f32(128, 128, false, false);
      const uint32_t idKV = idesc_bf16_f32(128, HD, false, true);
      const uint32_t idDQ = idesc_bf16_f32(128, HD, true, true);
      // descriptors built once; k-steps and stages are byte offsets (desc_add)
      auto kmaj = [](uint64_t d0, int kk) { return desc_add(d0, (uint32_t)((kk >> 2) * kChunkBytes + (kk & 3) * 32)); };
      auto mnmaj = [](uint64_t d0, int kk) { return desc_add(d0, (uint32_t)(kk * 2048)); };
      const uint64_t dK0 = desc_sw128(smem_u32(sK), 16, 1024), dK0mn = desc_sw128(smem_u32(sK), kChunkBytes, 1024);
      const uint64_t dV0 = desc_sw128(smem_u32(sV), 16, 1024);
      const uint64_t dQ0 = desc_sw128(smem_u32(sQ), 16, 1024), dQ0mn = desc_sw128(smem_u32(sQ), kChunkBytes, 1024);
      const uint64_t dO0 = desc_sw128(smem_u32(sDO), 16, 1024), dO0mn = desc_sw128(smem_u32(sDO), kChunkBytes, 1024);
      const uint64_t dPT = desc_sw128(smem_u32(sPT), 16, 1024);
      const uint64_t dDS = desc_sw128(smem_u32(sDST), 16, 1024), dDSmn = desc_sw128(smem_u32(sDST), kChunkBytes, 1024);
      uint64_t dK = dK0, dKmn = dK0mn, dV = dV0;  // this item's K/V stage
      int ni = 0, g0 = 0;  // items done, global iteration of this item's first tile
      // S^T = K Q^T and dP^T = V dO^T for the query tile of global iteration g (needs its Q/dO
      // stage and the previous S^T / dP^T read out of TMEM).
      auto issue_s = [&](int g) -> bool {
        const int st = g % STQ;
        if (!mbar_wait(&qdo_full[st], (uint32_t)((g / STQ) & 1), abort_flag, p.status, kErrWaitFull)) return false;
        if (!mbar_wait(s_empty, (uint32_t)(g & 1) ^ 1u, abort_flag, p.status, kErrWaitAccEmpty)) return false;
        BWD_TRACE(g, 0);
        tc_fence_after();
        const uint64_t q = desc_add(dQ0, (uint32_t)(st * L::kT)), dO = desc_add(dO0, (uint32_t)(st * L::kT));
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) umma_bf16_ss(tbase + cS, kmaj(dK, kk), kmaj(q, kk), idSS, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) umma_bf16_ss(tbase + cDP, kmaj(dV, kk), kmaj(dO, kk), idSS, kk > 0 ? 1u : 0u);
        umma_commit(s_full);
        return true;
      };
      // dV += P^T dO, dK += dS^T Q, dQ = dS K for global iteration g (`first`: the item's first tile).
      auto issue_grads = [&](int g, bool first) -> bool {
        const int st = g % STQ;
        const uint32_t par = (uint32_t)(g & 1);
        if (!mbar_wait(ds_full, par, abort_flag, p.status, kErrWaitAccum)) return false;
        BWD_TRACE(g, 1);
        // the previous item's dK / dV must be read out before this item's first tile overwrites them
        if (first && !mbar_wait(dkv_empty, (uint32_t)(ni & 1) ^ 1u, abort_flag, p.status, kErrWaitAccEmpty))
          return false;
        tc_fence_after();
        const uint64_t qmn = desc_add(dQ0mn, (uint32_t)(st * L::kT)), dOmn = desc_add(dO0mn, (uint32_t)(st * L::kT));
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          if constexpr (PT_TMEM)
            umma_bf16_ts(tbase + cDV, tbase + cPT + kk * 8, mnmaj(dOmn, kk), idKV, (!first || kk > 0) ? 1u : 0u);
          else
            umma_bf16_ss(tbase + cDV, kmaj(dPT, kk), mnmaj(dOmn, kk), idKV, (!first || kk > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          umma_bf16_ss(tbase + cDK, kmaj(dDS, kk), mnmaj(qmn, kk), idKV, (!first || kk > 0) ? 1u : 0u);
        const int qb = g % NDQB;
        if (!mbar_wait(&dq_empty[qb], (uint32_t)((g / NDQB) & 1) ^ 1u, abort_flag, p.status, kErrWaitAccEmpty))
          return false;
        BWD_TRACE(g, 2);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          umma_bf16_ss(tbase + cDQ + qb * HD, mnmaj(dDSmn, kk), mnmaj(dKmn, kk), idDQ, kk > 0 ? 1u : 0u);
        umma_commit(&dq_full[qb]);
        umma_commit(&qdo_empty[st]);
        umma_commit(ds_empty);
        return true;
      };
      bool ok = true;
      for (int r = 0; ok && r < rounds; ++r) {
        const int idx = bwd_item_index(r, ctas);
        if (idx >= n_items) continue;
        const BwdItem w = bwd_item(idx, nq, p.B, p.Hk, G, p.causal);
        const int ks = ni % KVST;
        if (!mbar_wait(&kv_full[ks], (uint32_t)((ni / KVST) & 1), abort_flag, p.status, kErrWaitFull)) break;
        dK = desc_add(dK0, (uint32_t)(ks * L::kT));
        dKmn = desc_add(dK0mn, (uint32_t)(ks * L::kT));
        dV = desc_add(dV0, (uint32_t)(ks * L::kT));
        if constexpr (HD == 64) {
          // software-pipelined: the next tile's S^T / dP^T run while the softmax
          // warps turn this tile's S^T / dP^T into P^T / dS^T
          if (w.n_it > 0) ok = issue_s(g0);
          for (int it = 0; ok && it < w.n_it; ++it) {
            if (it + 1 < w.n_it) ok = issue_s(g0 + it + 1);
            if (ok) ok = issue_grads(g0 + it, it == 0);
          }
        } else {
          // dQ shares S^T's TMEM columns: strictly in order
          for (int it = 0; ok && it < w.n_it; ++it) {
            ok = issue_s(g0 + it);
            if (ok) ok = issue_grads(g0 + it, it == 0);
          }
        }
        if (!ok) break;
        umma_commit(dkv_full);      // the epilogue may read this item's dK / dV
        umma_commit(&kv_empty[ks]); // the TMA warp may refill this K/V stage
        g0 += w.n_it;
        ++ni;
      }
      if (ni > 0) {  // every MMA has completed before the CTA can free TMEM
        volatile int no_abort = 0;
        mbar_wait(dkv_full, (uint32_t)((ni - 1) & 1), &no_abort, p.status, kErrWaitAccum);
      }
    }
    __syncwarp();
  } else if (warp < 2 + kBwdSoftmaxWarps) {
    // ---------------- softmax: thread r owns key row r; warpgroup g owns query columns [64g, 64g+64)
    const int g = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const float sc = p.scale_log2;
    bool ok = true;
    int gi = 0;
    for (int rr = 0; ok && rr < rounds; ++rr) {
      const int idx = bwd_item_index(rr, ctas);
      if (idx >= n_items) continue;
      const BwdItem w = bwd_item(idx, nq, p.B, p.Hk, G, p.causal);
      const int krow = w.kt * kTile + r;
      const bool key_dead = krow >= p.S;
      for (int it = 0; it < w.n_it; ++it, ++gi) {
        const int qt = w.qt0 + it % w.per_head;
        const int st = gi % STQ;
        const uint32_t par = (uint32_t)(gi & 1);
        if (!wait_lane0(&qdo_full[st], (uint32_t)((gi / STQ) & 1), abort_flag, p.status, kErrWaitFull) ||
            !wait_lane0(s_full, par, abort_flag, p.status, kErrWaitAccum)) {
          ok = false;
          break;
        }
        if (threadIdx.x == 64) BWD_TRACE(gi, 3);
        tc_fence_after();
        const bool mask = (p.causal && qt == w.kt) || key_dead;
        const float* lse2 = sLse + st * kTile;
        const float* dlt = sDelta + st * kTile;
        // Both 32-column chunks are computed into registers before waiting for the
        // previous tile's MMAs to release the P^T / dS^T tiles, so this tile's
        // exponentials overlap those MMAs.
        uint32_t pk[2][16], dk[2][16];
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          const int col0 = 64 * g + 32 * ch;
          float sv[32], dp[32];
          tmem_ld2_x32(tbase + lane_base + cS + col0, sv, tbase + lane_base + cDP + col0, dp);
          if (threadIdx.x == 64) BWD_TRACE(gi, 12 + 2 * ch);
          if (HD == 64 && ch == 1) {  // this warp's S^T / dP^T reads are done: next tile's MMAs may start
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_empty);
          }
          if (mask)
            bwd_softmax32<true, KP>(sv, dp, lse2 + col0, dlt + col0, sc, qt * kTile + col0, krow, key_dead, pk[ch],
                                dk[ch]);
          else
            bwd_softmax32<false, KP>(sv, dp, lse2 + col0, dlt + col0, sc, qt * kTile + col0, krow, key_dead, pk[ch],
                                 dk[ch]);
          if (threadIdx.x == 64) BWD_TRACE(gi, 13 + 2 * ch);
        }
        if (threadIdx.x == 64) BWD_TRACE(gi, 4);
        if (!wait_lane0(ds_empty, par ^ 1u, abort_flag, p.status, kErrWaitEmpty)) {
          ok = false;
          break;
        }
        if (threadIdx.x == 64) BWD_TRACE(gi, 5);
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          if constexpr (PT_TMEM)
            tmem_st_32x32b_x16_nowait(tbase + lane_base + cPT + (uint32_t)(32 * g + 16 * ch), pk[ch]);
          else
            store_row32_sw128(sPT, r, 2 * g + ch, pk[ch]);
          store_row32_sw128(sDST, r, 2 * g + ch, dk[ch]);
        }
        if constexpr (PT_TMEM) tmem_wait_st();
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(ds_full);
        if (threadIdx.x == 64) BWD_TRACE(gi, 6);
        if (threadIdx.x == 224) BWD_TRACE(gi, 11);
      }
    }
  } else {
    // ---------------- dQ warpgroup: drains each tile's dQ and writes each item's dK / dV.
    // Thread r owns TMEM lane r: query row r of the current q tile for dQ, key row r
    // of the item for dK / dV.  dQ goes TMEM -> registers -> SW128 fp32 staging tiles
    // in shared memory -> one bulk tensor reduce-add per 32 columns into the fp32
    // accumulator.  The dK / dV epilogue of an item overlaps the next item's softmax.
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const bool leader = threadIdx.x == (2 + kBwdSoftmaxWarps) * 32;
    constexpr int kDqThreads = 128, kDqBar = 1;
    // Only the leader waits on dq_full and publishes the outcome before the named
    // barrier, so every dQ warp takes the same path (a bar.sync has no timeout).
    volatile int* dq_ok = abort_flag + 1;
    constexpr int NCOL = HD / 32;            // 32-column chunks of a dQ row
    constexpr int NDQ = L::NDQ;              // chunks staged in shared memory at a time
    constexpr int NHOLD = NCOL - NDQ;        // chunks parked in registers until staging frees up
    bool ok = true;
    int gi = 0, ni = 0;
    for (int rr = 0; ok && rr < rounds; ++rr) {
      const int idx = bwd_item_index(rr, ctas);
      if (idx >= n_items) continue;
      const BwdItem w = bwd_item(idx, nq, p.B, p.Hk, G, p.causal);
      for (int it = 0; it < w.n_it; ++it, ++gi) {
        const int h = w.hk * G + it / w.per_head;
        const int qt = w.qt0 + it % w.per_head;
        const int qb = gi % NDQB;
        if (leader) {
          *dq_ok = mbar_wait(&dq_full[qb], (uint32_t)((gi / NDQB) & 1), abort_flag, p.status, kErrWaitAccum) ? 1 : 0;
          if (HD != 64) bulk_wait_read0();  // the previous tile's reduces have read the staging tiles
        }
        named_sync(kDqBar, kDqThreads);
        if (!*dq_ok) {
          ok = false;
          break;
        }
        if (leader) BWD_TRACE(gi, 7);
        tc_fence_after();
        const uint32_t src = tbase + lane_base + cDQ + qb * HD;
        if constexpr (HD == 64) {
          // the whole row into registers and the TMEM buffer released first; then the two
          // 32-column halves go through the one staging tile in turn
          float v[64];
          tmem_ld_32x32b_x64(src, v);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dq_empty[qb]);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            if (leader) bulk_wait_read0();  // the staging tile has been read by the previous reduce
            named_sync(kDqBar, kDqThreads);
            store_row_f32_sw128(sDQ, r, v + 32 * c);
            fence_proxy_async_smem();
            named_sync(kDqBar, kDqThreads);
            if (leader) {
              tma_reduce_add_3d(&tmDQ, sDQ, h * HD + 32 * c, qt * kTile, w.b);
              bulk_commit();
            }
          }
          if (leader) BWD_TRACE(gi, 8);
          continue;
        }
        float hold[NHOLD > 0 ? NHOLD * 32 : 1];
#pragma unroll
        for (int c = 0; c < NDQ; ++c) {
          float v[32];
          tmem_ld_32x32b_x32(src + c * 32, v);
          store_row_f32_sw128(sDQ + c * L::kDQ, r, v);
        }
#pragma unroll
        for (int c = 0; c < NHOLD; ++c) tmem_ld_32x32b_x32(src + (NDQ + c) * 32, hold + c * 32);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&dq_empty[qb]);
          if (HD != 64) mbar_arrive(s_empty);  // dQ shares S^T's TMEM columns
        }
#pragma unroll
        for (int c0 = 0; c0 < NCOL; c0 += NDQ) {
          if (c0 > 0) {  // stage the next chunks from registers once the staging tiles are read
            if (leader) bulk_wait_read0();
            named_sync(kDqBar, kDqThreads);
#pragma unroll
            for (int c = 0; c < NDQ; ++c) store_row_f32_sw128(sDQ + c * L::kDQ, r, hold + (c0 - NDQ + c) * 32);
          }
          fence_proxy_async_smem();
          named_sync(kDqBar, kDqThreads);
          if (leader) {
            for (int c = 0; c < NDQ; ++c)
              tma_reduce_add_3d(&tmDQ, sDQ + c * L::kDQ, h * HD + (c0 + c) * 32, qt * kTile, w.b);
            bulk_commit();
          }
        }
      }
      if (!ok) break;
      // epilogue of the item: dV, then dK (times the softmax scale), TMEM -> bf16 rows in global memory
      if (!wait_lane0(dkv_full, (uint32_t)(ni & 1), abort_flag, p.status, kErrWaitAccum)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int krow = w.kt * kTile + r;
      const bool key_dead = krow >= p.S;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        __nv_bfloat16* out = half == 0 ? p.dv + ((long)w.b * p.S + krow) * p.ld_dv + (long)w.hk * HD
                                       : p.dk + ((long)w.b * p.S + krow) * p.ld_dk + (long)w.hk * HD;
        const uint32_t col = tbase + lane_base + (half == 0 ? cDV : cDK);
        const float mul = half == 0 ? 1.f : p.scale;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          float v[32];
          tmem_ld_32x32b_x32(col + c * 32, v);
          if (half == 1 && c == HD / 32 - 1) {  // the last TMEM read of this item: MMAs may reuse dK / dV
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(dkv_empty);
          }
          if (!key_dead) {
#pragma unroll
            for (int i = 0; i < 32; i += 8)
              *reinterpret_cast<uint4*>(out + c * 32 + i) =
                  make_uint4(pack_bf16x2(v[i] * mul, v[i + 1] * mul), pack_bf16x2(v[i + 2] * mul, v[i + 3] * mul),
                             pack_bf16x2(v[i + 4] * mul, v[i + 5] * mul), pack_bf16x2(v[i + 6] * mul, v[i + 7] * mul));
          }
        }
      }
      ++ni;
    }
    if (leader) bulk_wait0();  // every reduce has landed before the CTA retires
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ backward, head dim 128
// Head dim 128 with 64-query tiles.  With 128-query tiles S^T, dP^T, dV and dK
// fill the 512 TMEM columns and dQ has to share S^T's, which serialises every
// iteration.  With 64 queries per tile:
//   S^T = K Q^T, dP^T = V dO^T   [128 keys x 64 q]   64 columns each
//   dQ^T = K^T dS^T              [128 dims x 64 q]   64 columns, two buffers
//   dV += P^T dO, dK += dS^T Q   [128 keys x 128 d] 128 columns each
// = 512 columns with nothing aliased, every MMA at M = 128.  dQ^T drains while
// the next tile's products run: thread d of the dQ warpgroup holds dimension d
// of 64 queries and writes them down the rows of a [64 q x 32 d] fp32 staging
// tile (a warp fills one 128-byte row per store: no bank conflicts), then bulk
// tensor reduce-adds (64-row boxes) go into the fp32 dQ accumulator.
// Shared memory: K, V (one stage, 64 KB), Q / dO (two stages of [64 x 128],
// 64 KB), P^T and dS^T ([128 x 64] each, 32 KB), dQ staging (32 KB), lse /
// delta rows.  Work items and roles are those of attn_bwd_kernel.
constexpr int kQ64 = 64;                    // query rows per tile
constexpr int kQ64Chunk = kQ64 * 128;       // [64 rows x 64 bf16] swizzled chunk
template <bool DQ>
struct BwdQ64Smem {
  static constexpr int HD = 128;
  static constexpr int STQ = 3;  // Q / dO stages: loads run two tiles ahead
  static constexpr int kKV = HD / 64 * kChunkBytes;     // [128 x 128] bf16
  static constexpr int kQT = HD / 64 * kQ64Chunk;       // [64 x 128] bf16
  static constexpr int kPT = kChunkBytes;               // [128 keys x 64 q] bf16
  static constexpr int kDQc = kQ64 * 128;               // [64 q x 32 fp32] staging chunk
  static constexpr int kBytes = 2 * kKV + 2 * STQ * kQT + 2 * kPT + (DQ ? HD / 32 : 0) * kDQc + 2 * STQ * kQ64 * 4;
};

__device__ __forceinline__ BwdItem bwd_item_q64(int idx, int nq64, int B, int Hk, int G, int causal) {
  BwdItem w;
  const int bh = idx % (B * Hk);
  w.kt = idx / (B * Hk);
  w.b = bh / Hk;
  w.hk = bh % Hk;
  w.qt0 = causal ? 2 * w.kt : 0;  // the first 64-query tile that sees key tile kt
  w.per_head = nq64 - w.qt0;
  w.n_it = G * w.per_head;
  return w;
}

template <int KP, bool DQ>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_q64_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                        const __grid_constant__ CUtensorMap tmDQ, const BwdParams p) {
  using L = BwdQ64Smem<DQ>;
  constexpr int HD = 128, STQ = L::STQ, NCH = HD / 64;
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t cS = 0, cDP = 64, cDQ = 128, cDV = 256, cDK = 384;  // dQ^T: two buffers of 64
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((base_u32 + 1023u) & ~1023u) - base_u32);
  uint8_t* sK = smem;
  uint8_t* sV = sK + L::kKV;
  uint8_t* sQ = sV + L::kKV;         // [STQ]
  uint8_t* sDO = sQ + STQ * L::kQT;  // [STQ]
  uint8_t* sPT = sDO + STQ * L::kQT;
  uint8_t* sDST = sPT + L::kPT;
  uint8_t* sDQ = sDST + L::kPT;                                     // HD/32 x [64 x 32] fp32
  float* sLse = reinterpret_cast<float*>(sDQ + (DQ ? HD / 32 : 0) * L::kDQc);  // [STQ][64]
  float* sDelta = sLse + STQ * kQ64;                                 // [STQ][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDelta + STQ * kQ64);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = kv_full + 1;
  uint64_t* qdo_full = kv_empty + 1;    // [STQ]
  uint64_t* qdo_empty = qdo_full + STQ; // [STQ]
  uint64_t* s_full = qdo_empty + STQ;
  uint64_t* s_empty = s_full + 1;       // every softmax warp has read S^T / dP^T
  uint64_t* ds_full = s_empty + 1;      // every softmax warp has stored P^T / dS^T
  uint64_t* ds_empty = ds_full + 1;     // the MMAs have read P^T / dS^T
  uint64_t* dq_full = ds_empty + 1;     // [2]
  uint64_t* dq_empty = dq_full + 2;     // [2]
  uint64_t* dkv_full = dq_empty + 2;
  uint64_t* dkv_empty = dkv_full + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(dkv_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (p.S + kTile - 1) / kTile;
  const int nq64 = (p.S + kQ64 - 1) / kQ64;
  const int G = p.Hq / p.Hk;
  const int n_items = nk * p.B * p.Hk;
  const int ctas = (int)gridDim.x;
  const int rounds = (n_items + ctas - 1) / ctas;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int s = 0; s < STQ; ++s) {
      mbar_init(&qdo_full[s], 2);  // the Q / dO copies, and the lse / delta rows
      mbar_init(&qdo_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, kBwdSoftmaxWarps);
    mbar_init(ds_full, kBwdSoftmaxWarps);
    mbar_init(ds_empty, 1);
    for (int j = 0; j < 2; ++j) {
      mbar_init(&dq_full[j], 1);
      mbar_init(&dq_empty[j], 4);
    }
    mbar_init(dkv_full, 1);
    mbar_init(dkv_empty, 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp == 0) {
    // ---------------- TMA warp: K/V per item, Q/dO (+ lse, delta rows) per 64-query tile
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmDO);
      tma_prefetch_desc(&tmDQ);
    }
    int ni = 0, gq = 0;
    bool ok = true;
    for (int r = 0; ok && r < rounds; ++r) {
      const int idx = bwd_item_index(r, ctas);
      if (idx >= n_items) continue;
      const BwdItem w = bwd_item_q64(idx, nq64, p.B, p.Hk, G, p.causal);
      if (!wait_lane0(kv_empty, (uint32_t)(ni & 1) ^ 1u, abort_flag, p.status, kErrWaitEmpty)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(kv_full, 2 * L::kKV);
        for (int c = 0; c < NCH; ++c) {
          tma_load_3d(sK + c * kChunkBytes, &tmK, kv_full, w.hk * HD + c * 64, w.kt * kTile, w.b);
          tma_load_3d(sV + c * kChunkBytes, &tmV, kv_full, w.hk * HD + c * 64, w.kt * kTile, w.b);
        }
      }
      ++ni;
      for (int it = 0; it < w.n_it; ++it, ++gq) {
        const int h = w.hk * G + it / w.per_head;
        const int qt = w.qt0 + it % w.per_head;
        const int st = gq % STQ;
        if (!wait_lane0(&qdo_empty[st], (uint32_t)((gq / STQ) & 1) ^ 1u, abort_flag, p.status, kErrWaitEmpty)) {
          ok = false;
          break;
        }
        if (lane == 0) {  // the bulk copies first, then the lse / delta rows while they fly
          mbar_arrive_expect_tx(&qdo_full[st], 2 * L::kQT);
          for (int c = 0; c < NCH; ++c) {
            tma_load_3d(sQ + st * L::kQT + c * kQ64Chunk, &tmQ, &qdo_full[st], h * HD + c * 64, qt * kQ64, w.b);
            tma_load_3d(sDO + st * L::kQT + c * kQ64Chunk, &tmDO, &qdo_full[st], h * HD + c * 64, qt * kQ64, w.b);
          }
        }
        const long row0 = ((long)w.b * p.Hq + h) * p.S;
        for (int i = lane; i < kQ64; i += 32) {
          const int q = qt * kQ64 + i;
          sLse[st * kQ64 + i] = q < p.S ? p.lse[row0 + q] * kLog2e : INFINITY;
          sDelta[st * kQ64 + i] = q < p.S ? p.delta[row0 + q] : 0.f;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&qdo_full[st]);
      }
    }
    if (lane == 0) {  // every bulk copy issued has landed before the CTA can retire
      volatile int no_abort = 0;
      if (ni > 0) mbar_wait(kv_full, (uint32_t)((ni - 1) & 1), &no_abort, p.status, kErrWaitFull);
      for (int g = gq - 1; g >= 0 && g >= gq - STQ; --g)
        mbar_wait(&qdo_full[g % STQ], (uint32_t)((g / STQ) & 1), &no_abort, p.status, kErrWaitFull);
    }
  } else if (warp == 1) {
    // ---------------- MMA warp
    if (elect_one()) {
      const uint32_t idS = idesc_bf16_f32(128, kQ64, false, false);   // S^T, dP^T: [128 keys x 64 q]
      const uint32_t idKV = idesc_bf16_f32(128, HD, false, true);     // dV, dK: [128 keys x 128 d]
      const uint32_t idDQ = idesc_bf16_f32(HD, kQ64, true, true);     // dQ^T: [128 d x 64 q]
      // K-major operand k-steps of 16: two 64-column chunks of the tile (chunk bytes differ by tile height)
      auto kmaj = [](uint64_t d0, int kk, uint32_t chunk) {
        return desc_add(d0, (uint32_t)((kk >> 2) * chunk + (kk & 3) * 32));
      };
      auto mnmaj = [](uint64_t d0, int kk) { return desc_add(d0, (uint32_t)(kk * 2048)); };
      const uint64_t dK = desc_sw128(smem_u32(sK), 16, 1024), dKmn = desc_sw128(smem_u32(sK), kChunkBytes, 1024);
      const uint64_t dV = desc_sw128(smem_u32(sV), 16, 1024);
      const uint64_t dQ0 = desc_sw128(smem_u32(sQ), 16, 1024), dQ0mn = desc_sw128(smem_u32(sQ), kQ64Chunk, 1024);
      const uint64_t dO0 = desc_sw128(smem_u32(sDO), 16, 1024), dO0mn = desc_sw128(smem_u32(sDO), kQ64Chunk, 1024);
      const uint64_t dPT = desc_sw128(smem_u32(sPT), 16, 1024);
      const uint64_t dDS = desc_sw128(smem_u32(sDST), 16, 1024), dDSmn = desc_sw128(smem_u32(sDST), kChunkBytes, 1024);
      int ni = 0, g0 = 0;
      auto issue_s = [&](int g) -> bool {
        const int st = g % STQ;
        if (!mbar_wait(&qdo_full[st], (uint32_t)((g / STQ) & 1), abort_flag, p.status, kErrWaitFull)) return false;
        if (!mbar_wait(s_empty, (uint32_t)(g & 1) ^ 1u, abort_flag, p.status, kErrWaitAccEmpty)) return false;
        tc_fence_after();
        const uint64_t q = desc_add(dQ0, (uint32_t)(st * L::kQT)), dO = desc_add(dO0, (uint32_t)(st * L::kQT));
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_bf16_ss(tbase + cS, kmaj(dK, kk, kChunkBytes), kmaj(q, kk, kQ64Chunk), idS, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_bf16_ss(tbase + cDP, kmaj(dV, kk, kChunkBytes), kmaj(dO, kk, kQ64Chunk), idS, kk > 0 ? 1u : 0u);
        umma_commit(s_full);
        return true;
      };
      auto issue_grads = [&](int g, bool first) -> bool {
        const int st = g % STQ;
        if (!mbar_wait(ds_full, (uint32_t)(g & 1), abort_flag, p.status, kErrWaitAccum)) return false;
        if (first && !mbar_wait(dkv_empty, (uint32_t)(ni & 1) ^ 1u, abort_flag, p.status, kErrWaitAccEmpty))
          return false;
        tc_fence_after();
        const uint64_t qmn = desc_add(dQ0mn, (uint32_t)(st * L::kQT)), dOmn = desc_add(dO0mn, (uint32_t)(st * L::kQT));
#pragma unroll
        for (int kk = 0; kk < kQ64 / 16; ++kk)
          umma_bf16_ss(tbase + cDV, kmaj(dPT, kk, kChunkBytes), mnmaj(dOmn, kk), idKV, (!first || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kQ64 / 16; ++kk)
          umma_bf16_ss(tbase + cDK, kmaj(dDS, kk, kChunkBytes), mnmaj(qmn, kk), idKV, (!first || kk > 0) ? 1u : 0u);
        if constexpr (DQ) {
          const int qb = g & 1;
          if (!mbar_wait(&dq_empty[qb], (uint32_t)((g >> 1) & 1) ^ 1u, abort_flag, p.status, kErrWaitAccEmpty))
            return false;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kTile / 16; ++kk)
            umma_bf16_ss(tbase + cDQ + qb * kQ64, mnmaj(dKmn, kk), mnmaj(dDSmn, kk), idDQ, kk > 0 ? 1u : 0u);
          umma_commit(&dq_full[qb]);
        }
        umma_commit(&qdo_empty[st]);
        umma_commit(ds_empty);
        return true;
      };
      bool ok = true;
      for (int r = 0; ok && r < rounds; ++r) {
        const int idx = bwd_item_index(r, ctas);
        if (idx >= n_items) continue;
        const BwdItem w = bwd_item_q64(idx, nq64, p.B, p.Hk, G, p.causal);
        if (!mbar_wait(kv_full, (uint32_t)(ni & 1), abort_flag, p.status, kErrWaitFull)) break;
        // software-pipelined: the next tile's S^T / dP^T run while the softmax warps
        // turn this tile's into P^T / dS^T
        if (w.n_it > 0) ok = issue_s(g0);
        for (int it = 0; ok && it < w.n_it; ++it) {
          if (it + 1 < w.n_it) ok = issue_s(g0 + it + 1);
          if (ok) ok = issue_grads(g0 + it, it == 0);
        }
        if (!ok) break;
        umma_commit(dkv_full);  // the epilogue may read this item's dK / dV
        umma_commit(kv_empty);  // the TMA warp may load the next item's K / V
        g0 += w.n_it;
        ++ni;
      }
      if (ni > 0) {  // every MMA has completed before the CTA can free TMEM
        volatile int no_abort = 0;
        mbar_wait(dkv_full, (uint32_t)((ni - 1) & 1), &no_abort, p.status, kErrWaitAccum);
      }
    }
    __syncwarp();
  } else if (warp < 2 + kBwdSoftmaxWarps) {
    // ---------------- softmax: thread r owns key row r; warpgroup t owns query columns [32t, 32t+32)
    const int t = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const float sc = p.scale_log2;
    const int col0 = 32 * t;
    bool ok = true;
    int gi = 0;
    for (int rr = 0; ok && rr < rounds; ++rr) {
      const int idx = bwd_item_index(rr, ctas);
      if (idx >= n_items) continue;
      const BwdItem w = bwd_item_q64(idx, nq64, p.B, p.Hk, G, p.causal);
      const int krow = w.kt * kTile + r;
      const bool key_dead = krow >= p.S;
      for (int it = 0; it < w.n_it; ++it, ++gi) {
        const int qt = w.qt0 + it % w.per_head;
        const int st = gi % STQ;
        const uint32_t par = (uint32_t)(gi & 1);
        if (!wait_lane0(&qdo_full[st], (uint32_t)((gi / STQ) & 1), abort_flag, p.status, kErrWaitFull) ||
            !wait_lane0(s_full, par, abort_flag, p.status, kErrWaitAccum)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // the two 64-query tiles that straddle the diagonal of key tile kt need the causal mask
        const bool mask = (p.causal && (qt >> 1) == w.kt) || key_dead;
        float sv[32], dp[32];
        tmem_ld2_x32(tbase + lane_base + cS + col0, sv, tbase + lane_base + cDP + col0, dp);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_empty);  // the next tile's S^T / dP^T may be computed
        uint32_t pk[16], dk[16];
        const float* lse2 = sLse + st * kQ64 + col0;
        const float* dlt = sDelta + st * kQ64 + col0;
        if (mask)
          bwd_softmax32<true, KP>(sv, dp, lse2, dlt, sc, qt * kQ64 + col0, krow, key_dead, pk, dk);
        else
          bwd_softmax32<false, KP>(sv, dp, lse2, dlt, sc, qt * kQ64 + col0, krow, key_dead, pk, dk);
        if (!wait_lane0(ds_empty, par ^ 1u, abort_flag, p.status, kErrWaitEmpty)) {
          ok = false;
          break;
        }
        store_row32_sw128(sPT, r, t, pk);
        store_row32_sw128(sDST, r, t, dk);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ds_full);
      }
    }
  } else {
    // ---------------- dQ warpgroup: drains each tile's dQ^T and writes each item's dK / dV.
    // Thread r owns TMEM lane r: head dimension r for dQ^T, key row r for dK / dV.
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const bool leader = threadIdx.x == (2 + kBwdSoftmaxWarps) * 32;
    constexpr int kDqThreads = 128, kDqBar = 1;
    volatile int* dq_ok = abort_flag + 1;
    // dimension r lands in staging chunk r / 32 (= this warp's), column r % 32: byte
    // offset of 16-byte unit (r % 32) / 4, swizzled by the row (query) within 8
    uint8_t* my_chunk = sDQ + (r >> 5) * L::kDQc;
    const int unit = (r & 31) >> 2, within = (r & 3) * 4;
    bool ok = true;
    int gi = 0, ni = 0;
    for (int rr = 0; ok && rr < rounds; ++rr) {
      const int idx = bwd_item_index(rr, ctas);
      if (idx >= n_items) continue;
      const BwdItem w = bwd_item_q64(idx, nq64, p.B, p.Hk, G, p.causal);
      for (int it = 0; DQ && it < w.n_it; ++it, ++gi) {
        const int h = w.hk * G + it / w.per_head;
        const int qt = w.qt0 + it % w.per_head;
        const int qb = gi & 1;
        if (leader) {
          *dq_ok = mbar_wait(&dq_full[qb], (uint32_t)((gi >> 1) & 1), abort_flag, p.status, kErrWaitAccum) ? 1 : 0;
          bulk_wait_read0();  // the previous tile's reduce-adds have read the staging tile
        }
        named_sync(kDqBar, kDqThreads);
        if (!*dq_ok) {
          ok = false;
          break;
        }
        tc_fence_after();
        float v0[32], v1[32];
        tmem_ld2_x32(tbase + lane_base + cDQ + qb * kQ64, v0, tbase + lane_base + cDQ + qb * kQ64 + 32, v1);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dq_empty[qb]);  // the next-but-one tile's dQ^T may be computed
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          *reinterpret_cast<float*>(my_chunk + q * 128 + ((unit ^ (q & 7)) << 4) + within) = v0[q];
          *reinterpret_cast<float*>(my_chunk + (q + 32) * 128 + ((unit ^ (q & 7)) << 4) + within) = v1[q];
        }
        fence_proxy_async_smem();
        named_sync(kDqBar, kDqThreads);
        if (leader) {
          for (int c = 0; c < HD / 32; ++c)
            tma_reduce_add_3d(&tmDQ, sDQ + c * L::kDQc, h * HD + 32 * c, qt * kQ64, w.b);
          bulk_commit();
        }
      }
      if (!ok) break;
      // epilogue of the item: dV, then dK (times the softmax scale), TMEM -> bf16 rows in global memory
      if (!wait_lane0(dkv_full, (uint32_t)(ni & 1), abort_flag, p.status, kErrWaitAccum)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int krow = w.kt * kTile + r;
      const bool key_dead = krow >= p.S;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        __nv_bfloat16* out = half == 0 ? p.dv + ((long)w.b * p.S + krow) * p.ld_dv + (long)w.hk * HD
                                       : p.dk + ((long)w.b * p.S + krow) * p.ld_dk + (long)w.hk * HD;
        const uint32_t col = tbase + lane_base + (half == 0 ? cDV : cDK);
        const float mul = half == 0 ? 1.f : p.scale;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          float v[32];
          tmem_ld_32x32b_x32(col + c * 32, v);
          if (half == 1 && c == HD / 32 - 1) {  // the last TMEM read of this item: MMAs may reuse dK / dV
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(dkv_empty);
          }
          if (!key_dead) {
#pragma unroll
            for (int i = 0; i < 32; i += 8)
              *reinterpret_cast<uint4*>(out + c * 32 + i) =
                  make_uint4(pack_bf16x2(v[i] * mul, v[i + 1] * mul), pack_bf16x2(v[i + 2] * mul, v[i + 3] * mul),
                             pack_bf16x2(v[i + 4] * mul, v[i + 5] * mul), pack_bf16x2(v[i + 6] * mul, v[i + 7] * mul));
          }
        }
      }
      ++ni;
    }
    if (DQ && leader) bulk_wait0();  // every reduce has landed before the CTA retires
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ backward, dQ pass (query-stationary)
// dQ without atomics: one CTA per (query tile, head) walks its key tiles and
// accumulates dQ in TMEM, recomputing S and dP (two more products than the
// key-stationary pass, which then computes dK and dV only).  Per key tile j:
//   S = Q K_j^T, dP = dO V_j^T                  [128 q x 128 keys]  TMEM
//   dS = P (dP - delta), P = 2^(S sc - lse)     softmax warps, thread = query row
//   dQ += dS K_j                                [128 q x HD]        TMEM
// dS goes to shared memory as the A operand (K-major); K_j is the MN-major B
// operand.  S_{j+1} / dP_{j+1} are issued as soon as the softmax warps have
// read S_j / dP_j, so the tensor core overlaps the softmax; the K/V ring keeps
// K_j until dQ += dS_j K_j has read it.  The epilogue scales dQ and writes it
// as bf16: no fp32 accumulator, no clearing, no conversion pass.
template <int HD>
struct BwdDqSmem {
  static constexpr int ST = HD == 64 ? 3 : 2;        // K/V stages
  static constexpr int kT = HD / 64 * kChunkBytes;   // one [128 x HD] bf16 tile
  static constexpr int kDS = 2 * kChunkBytes;        // [128 q x 128 keys] bf16
  static constexpr int kBytes = 2 * kT + 2 * ST * kT + kDS;
};
constexpr int kBwdDqThreads = 320;
constexpr int kMaxDynSmem = 232448;  // 227 KB per CTA
static_assert(BwdDqSmem<128>::kBytes + 1024 + 256 <= kMaxDynSmem, "dQ pass exceeds shared memory");
static_assert(BwdQ64Smem<true>::kBytes + 1024 + 256 <= kMaxDynSmem, "64-query pass exceeds shared memory");
static_assert(BwdSmem<64>::kBytes + 1024 + 256 <= kMaxDynSmem, "backward exceeds shared memory");

// dS = 2^(s sc - lse) (dp - delta) for 32 key columns of one query row, as bf16
// pairs.  MASK: keys past lim (causal diagonal, or past the sequence) give 0.
template <bool MASK, int KP>
__device__ __forceinline__ void dq_softmax32(const float* sv, const float* dp, float sc, float neg_lse, float dlt,
                                             int lim, uint32_t* out) {
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const int j = 2 * q;
    float e0, e1;
    if (!MASK && KP > 0 && poly_pair<KP>(q)) {
      f2unpack(ex2_poly_x2(fma_f32x2(f2pack(sv[j], sv[j + 1]), f2pack(sc, sc), f2pack(neg_lse, neg_lse))), e0, e1);
    } else {
      e0 = ex2_approx(fmaf(sv[j], sc, neg_lse));
      e1 = ex2_approx(fmaf(sv[j + 1], sc, neg_lse));
      if (MASK) {
        if (j >= lim) e0 = 0.f;
        if (j + 1 >= lim) e1 = 0.f;
      }
    }
    out[q] = pack_bf16x2(e0 * (dp[j] - dlt), e1 * (dp[j + 1] - dlt));
  }
}

template <int HD, int KP>
__global__ void __launch_bounds__(kBwdDqThreads, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const BwdParams p, __nv_bfloat16* __restrict__ dq, long ld_dq) {
  using L = BwdDqSmem<HD>;
  constexpr int ST = L::ST, NCH = HD / 64;
  constexpr uint32_t TMEM_COLS = 512, cS = 0, cDP = 128, cDQ = 256;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((base_u32 + 1023u) & ~1023u) - base_u32);
  uint8_t* sQ = smem;
  uint8_t* sDO = sQ + L::kT;
  uint8_t* sK = sDO + L::kT;        // [ST]
  uint8_t* sV = sK + ST * L::kT;    // [ST]
  uint8_t* sDS = sV + ST * L::kT;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDS + L::kDS);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;     // [ST]
  uint64_t* kv_empty = kv_full + ST;  // [ST]
  uint64_t* s_full = kv_empty + ST;
  uint64_t* s_empty = s_full + 1;     // every softmax warp has read S / dP
  uint64_t* ds_full = s_empty + 1;    // every softmax warp has stored its dS
  uint64_t* ds_empty = ds_full + 1;   // dQ += dS K has read dS
  uint64_t* dq_done = ds_empty + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(dq_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (p.S + kTile - 1) / kTile;
  const int qt = nq - 1 - (int)blockIdx.x;  // heaviest causal tiles first
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hk = h / (p.Hq / p.Hk);
  const int n_kv = p.causal ? qt + 1 : nq;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 8);
    mbar_init(ds_full, 8);
    mbar_init(ds_empty, 1);
    mbar_init(dq_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmDO);
      mbar_arrive_expect_tx(q_full, 2 * L::kT);
      for (int c = 0; c < NCH; ++c) {
        tma_load_3d(sQ + c * kChunkBytes, &tmQ, q_full, h * HD + c * 64, qt * kTile, b);
        tma_load_3d(sDO + c * kChunkBytes, &tmDO, q_full, h * HD + c * 64, qt * kTile, b);
      }
      int armed = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % ST;
        if (!mbar_wait(&kv_empty[st], (uint32_t)((j / ST) & 1) ^ 1u, abort_flag, p.status, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * L::kT);
        for (int c = 0; c < NCH; ++c) {
          tma_load_3d(sK + st * L::kT + c * kChunkBytes, &tmK, &kv_full[st], hk * HD + c * 64, j * kTile, b);
          tma_load_3d(sV + st * L::kT + c * kChunkBytes, &tmV, &kv_full[st], hk * HD + c * 64, j * kTile, b);
        }
        armed = j + 1;
      }
      volatile int no_abort = 0;  // every bulk copy issued has landed before the CTA can retire
      mbar_wait(q_full, 0, &no_abort, p.status, kErrWaitFull);
      for (int j = armed - 1; j >= 0 && j >= armed - ST; --j)
        mbar_wait(&kv_full[j % ST], (uint32_t)((j / ST) & 1), &no_abort, p.status, kErrWaitFull);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idS = idesc_bf16_f32(128, 128, false, false);
      const uint32_t idDQ = idesc_bf16_f32(128, HD, false, true);
      auto kmaj = [](uint64_t d0, int kk) { return desc_add(d0, (uint32_t)((kk >> 2) * kChunkBytes + (kk & 3) * 32)); };
      auto mnmaj = [](uint64_t d0, int kk) { return desc_add(d0, (uint32_t)(kk * 2048)); };
      const uint64_t dQd = desc_sw128(smem_u32(sQ), 16, 1024), dOd = desc_sw128(smem_u32(sDO), 16, 1024);
      const uint64_t dK0 = desc_sw128(smem_u32(sK), 16, 1024), dK0mn = desc_sw128(smem_u32(sK), kChunkBytes, 1024);
      const uint64_t dV0 = desc_sw128(smem_u32(sV), 16, 1024);
      const uint64_t dDS = desc_sw128(smem_u32(sDS), 16, 1024);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, kErrWaitFull);
      // dQ += dS_j K_j once the softmax warps have stored dS_j
      auto issue_dq = [&](int j) -> bool {
        if (!mbar_wait(ds_full, (uint32_t)(j & 1), abort_flag, p.status, kErrWaitAccum)) return false;
        tc_fence_after();
        const uint64_t kmn = desc_add(dK0mn, (uint32_t)((j % ST) * L::kT));
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          umma_bf16_ss(tbase + cDQ, kmaj(dDS, kk), mnmaj(kmn, kk), idDQ, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(ds_empty);
        umma_commit(&kv_empty[j % ST]);
        return true;
      };
      for (int j = 0; ok && j < n_kv; ++j) {
        const int st = j % ST;
        if (!mbar_wait(&kv_full[st], (uint32_t)((j / ST) & 1), abort_flag, p.status, kErrWaitFull)) {
          ok = false;
          break;
        }
        // S_j / dP_j overwrite S_{j-1} / dP_{j-1} once every softmax warp has read them
        if (!mbar_wait(s_empty, (uint32_t)(j & 1) ^ 1u, abort_flag, p.status, kErrWaitAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t kd = desc_add(dK0, (uint32_t)(st * L::kT)), vd = desc_add(dV0, (uint32_t)(st * L::kT));
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) umma_bf16_ss(tbase + cS, kmaj(dQd, kk), kmaj(kd, kk), idS, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) umma_bf16_ss(tbase + cDP, kmaj(dOd, kk), kmaj(vd, kk), idS, kk > 0 ? 1u : 0u);
        umma_commit(s_full);
        if (j > 0) ok = issue_dq(j - 1);
      }
      if (ok && n_kv > 0) issue_dq(n_kv - 1);
      umma_commit(dq_done);
      volatile int no_abort = 0;
      mbar_wait(dq_done, 0, &no_abort, p.status, kErrWaitAccum);
    }
    __syncwarp();
  } else {
    // ---------------- softmax: thread r owns query row r; warpgroup g owns key columns [64g, 64g+64)
    const int g = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const int qrow = qt * kTile + r;
    const float sc = p.scale_log2;
    const long row0 = ((long)b * p.Hq + h) * p.S;
    const float lse2 = qrow < p.S ? p.lse[row0 + qrow] * kLog2e : INFINITY;
    const float dlt = qrow < p.S ? p.delta[row0 + qrow] : 0.f;
    const float neg_lse = -lse2;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!wait_lane0(s_full, (uint32_t)(j & 1), abort_flag, p.status, kErrWaitAccum)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t pk[2][16];
      const bool diag = p.causal && j == qt;
      const bool tail = j * kTile + kTile > p.S;
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        const int col0 = 64 * g + 32 * ch;
        float sv[32], dp[32];
        tmem_ld2_x32(tbase + lane_base + cS + col0, sv, tbase + lane_base + cDP + col0, dp);
        if (ch == 1) {  // this warp's S / dP reads are done: the next tile's S / dP may start
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(s_empty);
        }
        if (diag || tail) {
          // keys past lim give 0: the causal diagonal (key > query) and keys past the sequence
          const int kmax = min(p.S, diag ? qrow + 1 : p.S) - (j * kTile + col0);
          dq_softmax32<true, KP>(sv, dp, sc, neg_lse, dlt, kmax, pk[ch]);
        } else {
          dq_softmax32<false, KP>(sv, dp, sc, neg_lse, dlt, 32, pk[ch]);
        }
      }
      if (!wait_lane0(ds_empty, (uint32_t)(j & 1) ^ 1u, abort_flag, p.status, kErrWaitEmpty)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) store_row32_sw128(sDS, r, 2 * g + ch, pk[ch]);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
    }
    // epilogue: dQ (times the softmax scale) -> bf16 rows; warpgroup g writes columns [g HD/2, (g+1) HD/2)
    if (ok && n_kv > 0 && wait_lane0(dq_done, 0, abort_flag, p.status, kErrWaitAccum)) {
      tc_fence_after();
      __nv_bfloat16* out = dq + ((long)b * p.S + qrow) * ld_dq + (long)h * HD;
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
        const int col = g * (HD / 2) + 32 * c;
        float v[32];
        tmem_ld_32x32b_x32(tbase + lane_base + cDQ + col, v);
        if (qrow < p.S) {
#pragma unroll
          for (int i = 0; i < 32; i += 8)
            *reinterpret_cast<uint4*>(out + col + i) = make_uint4(
                pack_bf16x2(v[i] * p.scale, v[i + 1] * p.scale), pack_bf16x2(v[i + 2] * p.scale, v[i + 3] * p.scale),
                pack_bf16x2(v[i + 4] * p.scale, v[i + 5] * p.scale), pack_bf16x2(v[i + 6] * p.scale, v[i + 7] * p.scale));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

// delta[b,h,q] = sum_d dO * O: one thread per (b, q, h) row, 16-byte loads;
// consecutive threads read consecutive heads of a token (contiguous bytes).
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ dout, long ld_do,
                                  const __nv_bfloat16* __restrict__ o, long ld_o, float* __restrict__ delta, int B,
                                  int S, int Hq, int HD) {
  const long row = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= (long)B * S * Hq) return;
  const int h = (int)(row % Hq);
  const long bs = row / Hq;
  const int s = (int)(bs % S), b = (int)(bs / S);
  const uint4* a = reinterpret_cast<const uint4*>(dout + bs * ld_do + (long)h * HD);
  const uint4* c = reinterpret_cast<const uint4*>(o + bs * ld_o + (long)h * HD);
  float acc = 0.f;
  for (int i = 0; i < HD / 8; ++i) {
    const uint4 x = a[i], y = c[i];
    const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fx = unpack_bf16x2(xs[j]), fy = unpack_bf16x2(ys[j]);
      acc = fmaf(fx.x, fy.x, fmaf(fx.y, fy.y, acc));
    }
  }
  delta[((long)b * Hq + h) * S + s] = acc;
}

// dq[b,s,h,:] = bf16(dq_accum * scale)
__global__ void attn_dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, long ld_dq,
                                       int B, int S, int Hq, int HD, float scale) {
  const long idx = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const long total = (long)B * S * Hq * HD;
  if (idx >= total) return;
  const int d = (int)(idx % HD);
  const long rh = idx / HD;
  const int h = (int)(rh % Hq);
  const long bs = rh / Hq;
  const float4 a = *reinterpret_cast<const float4*>(acc + idx);
  const float4 c = *reinterpret_cast<const float4*>(acc + idx + 4);
  *reinterpret_cast<uint4*>(dq + bs * ld_dq + (long)h * HD + d) =
      make_uint4(pack_bf16x2(a.x * scale, a.y * scale), pack_bf16x2(a.z * scale, a.w * scale),
                 pack_bf16x2(c.x * scale, c.y * scale), pack_bf16x2(c.z * scale, c.w * scale));
}

// ------------------------------------------------------------------ host side

static PFN_cuTensorMapEncodeTiled_v12000 attn_encode_fn() {
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

// {cols, S, B} map over rows of width ld (elements); box {64, 128, 1}.
static bool make_map3(CUtensorMap* m, const void* ptr, long cols, long S, long B, long ld, int box_rows = kTile) {
  auto fn = attn_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(S * ld * 2)};
  cuuint32_t box[3] = {64u, (cuuint32_t)box_rows, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// fp32 accumulator [B, S, cols] (rows of exactly `cols` floats); box {32, box_rows, 1},
// 128-byte swizzle: the target of the backward's bulk reduce-add of dQ.
static bool make_map3_f32(CUtensorMap* m, float* ptr, long cols, long S, long B, int box_rows = kTile) {
  auto fn = attn_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)(cols * 4), (cuuint64_t)(S * cols * 4)};
  cuuint32_t box[3] = {32u, (cuuint32_t)box_rows, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename K>
static void set_smem(K kern, int bytes) {
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// The dynamic shared-memory limit is a per-device attribute of a kernel: set
// it once for each device a process launches on.  `Id` names the kernel, since
// two instantiations with one signature share a function-pointer type.
template <int Id, typename K>
static void set_smem_once(K kern, int bytes, int device) {
  static std::once_flag flags[64];
  std::call_once(flags[device & 63], [&] { set_smem(kern, bytes); });
}

// Streaming multiprocessors of a device (read once per device).
static int sm_count(int device) {
  static int counts[64] = {0};
  int& n = counts[device & 63];
  if (n == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
    n = v;
  }
  return n;
}

// The persistent backward runs one CTA per SM (it holds all 512 TMEM columns).
static dim3 bwd_grid(int S, int B, int Hk, int device) {
  const long items = (long)((S + kTile - 1) / kTile) * B * Hk;
  return dim3((unsigned)std::max(1L, std::min(items, (long)sm_count(device))));
}

// Share of the softmax exponentials computed on the FMA pipe, in column pairs of
// 16: compiled defaults, overridable for tuning by MT_ATTN_POLY="fwd,bwd"
// (forward 0/4/6/8, backward 0/3/5/7; other values fall back to the defaults).
struct PolyShare {
  int fwd = kFwdPolyPairs, bwd = kBwdPolyPairs;
};
static const PolyShare& poly_share() {
  static const PolyShare share = [] {
    PolyShare ps;
    if (const char* env = getenv("MT_ATTN_POLY")) {
      int f = -1, b = -1;
      if (sscanf(env, "%d,%d", &f, &b) == 2) {
        ps.fwd = f;
        ps.bwd = b;
      }
    }
    return ps;
  }();
  return share;
}

// Forward kernel per head dim (measured on B200, CUDA events): head dim 64 runs the
// two-tile kernel with both warpgroups in step (110 us against 129 us for the
// ping-pong kernel at B4 S2048 H20), head dim 128 the ping-pong kernel (203 us
// against 216 us for the one-tile kernel at B1 S4096 Hq32 Hk8).  MT_ATTN_FWD=pp
// or =legacy forces one family for both.
static bool fwd_use_pingpong(int hd) {
  static const int forced = [] {
    const char* env = getenv("MT_ATTN_FWD");
    if (env && strcmp(env, "pp") == 0) return 1;
    if (env && strcmp(env, "legacy") == 0) return 0;
    return -1;
  }();
  return forced >= 0 ? forced == 1 : hd == 128;
}

// Alternating exponential phases in the ping-pong forward (MT_ATTN_ALT=1); off by
// default: measured about 4 % slower at head dim 128 than letting the warpgroups drift.
static int fwd_alternate() {
  static const int alt = [] {
    const char* env = getenv("MT_ATTN_ALT");
    return env ? atoi(env) : 0;
  }();
  return alt;
}

// Backward at head dim 128 (MT_ATTN_BWD, for A/B).  "q64" (default): one key-stationary
// pass on 64-query tiles with dQ reduce-adds, 457 us at B1 S4096 Hq32 Hk8; "split": that
// pass for dK / dV plus a query-stationary dQ pass (606 us: the recomputed products cost
// more than the reduce-adds they remove); "legacy": the 128-query pass with dQ sharing
// S^T's TMEM columns (872 us).
enum { kBwdOne = 0, kBwdQ64 = 1, kBwdSplit = 2 };
static int bwd_mode_hd128() {
  static const int mode = [] {
    const char* env = getenv("MT_ATTN_BWD");
    if (env && strcmp(env, "legacy") == 0) return (int)kBwdOne;
    if (env && strcmp(env, "split") == 0) return (int)kBwdSplit;
    return (int)kBwdQ64;
  }();
  return mode;
}

static int check_args(const AttnArgs& a, char* err, int errlen) {
  if (a.hd != 64 && a.hd != 128) {
    snprintf(err, errlen, "attention: head_dim %d unsupported (64 or 128)", a.hd);
    return -1;
  }
  if (a.Hk <= 0 || a.Hq % a.Hk) {
    snprintf(err, errlen, "attention: Hq (%d) must be a multiple of Hk (%d)", a.Hq, a.Hk);
    return -1;
  }
  if ((a.ld_q | a.ld_k | a.ld_v | a.ld_o) & 7) {
    snprintf(err, errlen, "attention: row strides must be multiples of 8 elements");
    return -1;
  }
  return 0;
}

int attention_fwd(const AttnArgs& a, int device, cudaStream_t s, char* err, int errlen) {
  if (check_args(a, err, errlen)) return -1;
  if (a.B == 0 || a.S == 0) return 0;
  CUtensorMap mq, mk, mv;
  if (!make_map3(&mq, a.q, (long)a.Hq * a.hd, a.S, a.B, a.ld_q) || !make_map3(&mk, a.k, (long)a.Hk * a.hd, a.S, a.B, a.ld_k) ||
      !make_map3(&mv, a.v, (long)a.Hk * a.hd, a.S, a.B, a.ld_v)) {
    snprintf(err, errlen, "attention: tensor map encode failed");
    return -1;
  }
  FwdParams p{};
  p.o = reinterpret_cast<__nv_bfloat16*>(a.o);
  p.ld_o = a.ld_o;
  p.lse = a.lse;
  p.B = a.B;
  p.S = a.S;
  p.Hq = a.Hq;
  p.Hk = a.Hk;
  p.scale_log2 = a.scale * kLog2e;
  p.causal = a.causal ? 1 : 0;
  p.status = device_status(device);
  p.alternate = fwd_alternate();
  const int nq = (a.S + kTile - 1) / kTile;
  dim3 grid(nq, a.B * a.Hq);
  const int barrier_bytes = 256;
  const int kp = poly_share().fwd;
  if (fwd_use_pingpong(a.hd)) {
    const dim3 g2((nq + 1) / 2, a.B * a.Hq);
    auto go = [&](auto kern, int smem, auto id) {
      set_smem_once<decltype(id)::value>(kern, smem, device);
      kern<<<g2, kFwdPPThreads, smem, s>>>(mq, mk, mv, p);
    };
    if (a.hd == 64) {
      constexpr int smem = FwdPPSmem<64>::kBytes + 1024 + barrier_bytes;
      if (kp == 0) go(attn_fwd_pp_kernel<64, 0>, smem, std::integral_constant<int, 20>{});
      else if (kp == 4) go(attn_fwd_pp_kernel<64, 4>, smem, std::integral_constant<int, 21>{});
      else if (kp == 8) go(attn_fwd_pp_kernel<64, 8>, smem, std::integral_constant<int, 22>{});
      else go(attn_fwd_pp_kernel<64, kFwdPolyPairs>, smem, std::integral_constant<int, 23>{});
    } else {
      constexpr int smem = FwdPPSmem<128>::kBytes + 1024 + barrier_bytes;
      if (kp == 0) go(attn_fwd_pp_kernel<128, 0>, smem, std::integral_constant<int, 24>{});
      else if (kp == 4) go(attn_fwd_pp_kernel<128, 4>, smem, std::integral_constant<int, 25>{});
      else if (kp == 8) go(attn_fwd_pp_kernel<128, 8>, smem, std::integral_constant<int, 26>{});
      else go(attn_fwd_pp_kernel<128, kFwdPolyPairs>, smem, std::integral_constant<int, 27>{});
    }
  } else if (a.hd == 64) {
    constexpr int smem = Fwd2QSmem::kBytes + 1024 + barrier_bytes;
    const dim3 g2((nq + 1) / 2, a.B * a.Hq);
    auto go = [&](auto kern, auto id) {
      set_smem_once<decltype(id)::value>(kern, smem, device);
      kern<<<g2, kFwd2QThreads, smem, s>>>(mq, mk, mv, p);
    };
    if (kp == 0) go(attn_fwd_2q_kernel<0>, std::integral_constant<int, 0>{});
    else if (kp == 4) go(attn_fwd_2q_kernel<4>, std::integral_constant<int, 4>{});
    else if (kp == 8) go(attn_fwd_2q_kernel<8>, std::integral_constant<int, 5>{});
    else go(attn_fwd_2q_kernel<kFwdPolyPairs>, std::integral_constant<int, 6>{});
  } else {
    constexpr int smem = FwdSmem<128, 3>::kBytes + 1024 + barrier_bytes;
    auto go = [&](auto kern, auto id) {
      set_smem_once<decltype(id)::value>(kern, smem, device);
      kern<<<grid, 192, smem, s>>>(mq, mk, mv, p);
    };
    if (kp == 0) go(attn_fwd_kernel<128, 3, 0>, std::integral_constant<int, 1>{});
    else if (kp == 4) go(attn_fwd_kernel<128, 3, 4>, std::integral_constant<int, 7>{});
    else if (kp == 8) go(attn_fwd_kernel<128, 3, 8>, std::integral_constant<int, 8>{});
    else go(attn_fwd_kernel<128, 3, kFwdPolyPairs>, std::integral_constant<int, 9>{});
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(err, errlen, "attention_fwd launch: %s", cudaGetErrorString(e));
    return (int)e;
  }
  return 0;
}

int attention_bwd(const AttnBwdArgs& a, int device, cudaStream_t s, char* err, int errlen) {
  const AttnArgs& f = a.f;
  if (check_args(f, err, errlen)) return -1;
  if ((a.ld_do | a.ld_dq | a.ld_dk | a.ld_dv) & 7) {
    snprintf(err, errlen, "attention_bwd: row strides must be multiples of 8 elements");
    return -1;
  }
  if (f.B == 0 || f.S == 0) return 0;
  const long rows = (long)f.B * f.S * f.Hq;
  // head dim 128: 64-query tiles for the key-stationary pass (dQ by reduce-adds, or in
  // its own query-stationary pass in the split mode)
  const int mode = f.hd == 128 ? bwd_mode_hd128() : kBwdOne;
  const bool split = mode == kBwdSplit;
  const int qrows = mode == kBwdOne ? kTile : kQ64;
  if (!split) cudaMemsetAsync(a.dq_accum, 0, rows * f.hd * sizeof(float), s);
  attn_delta_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(a.dout), a.ld_do, reinterpret_cast<const __nv_bfloat16*>(f.o), f.ld_o,
      a.delta, f.B, f.S, f.Hq, f.hd);
  CUtensorMap mq, mk, mv, mdo, mdq;
  if (!make_map3(&mq, f.q, (long)f.Hq * f.hd, f.S, f.B, f.ld_q, qrows) ||
      !make_map3(&mk, f.k, (long)f.Hk * f.hd, f.S, f.B, f.ld_k) ||
      !make_map3(&mv, f.v, (long)f.Hk * f.hd, f.S, f.B, f.ld_v) ||
      !make_map3(&mdo, a.dout, (long)f.Hq * f.hd, f.S, f.B, a.ld_do, qrows) ||
      (!split && !make_map3_f32(&mdq, a.dq_accum, (long)f.Hq * f.hd, f.S, f.B, qrows))) {
    snprintf(err, errlen, "attention_bwd: tensor map encode failed");
    return -1;
  }
  if (split) mdq = mq;  // unused by the pass without dQ
  BwdParams p{};
  p.lse = f.lse;
  p.delta = a.delta;
  p.dk = reinterpret_cast<__nv_bfloat16*>(a.dk);
  p.dv = reinterpret_cast<__nv_bfloat16*>(a.dv);
  p.ld_dk = a.ld_dk;
  p.ld_dv = a.ld_dv;
  p.B = f.B;
  p.S = f.S;
  p.Hq = f.Hq;
  p.Hk = f.Hk;
  p.scale_log2 = f.scale * kLog2e;
  p.scale = f.scale;
  p.causal = f.causal ? 1 : 0;
  p.status = device_status(device);
  const dim3 grid = bwd_grid(f.S, f.B, f.Hk, device);
  const int barrier_bytes = 256;
  const int kp = poly_share().bwd;
  auto go = [&](auto kern, int smem, auto id) {
    set_smem_once<decltype(id)::value>(kern, smem, device);
    kern<<<grid, kBwdThreads, smem, s>>>(mq, mk, mv, mdo, mdq, p);
  };
  if (f.hd == 64) {
    constexpr int smem = BwdSmem<64>::kBytes + 1024 + barrier_bytes;
    if (kp == 0) go(attn_bwd_kernel<64, 0>, smem, std::integral_constant<int, 10>{});
    else if (kp == 3) go(attn_bwd_kernel<64, 3>, smem, std::integral_constant<int, 11>{});
    else if (kp == 7) go(attn_bwd_kernel<64, 7>, smem, std::integral_constant<int, 12>{});
    else go(attn_bwd_kernel<64, kBwdPolyPairs>, smem, std::integral_constant<int, 2>{});
  } else if (mode == kBwdQ64) {
    constexpr int smem = BwdQ64Smem<true>::kBytes + 1024 + barrier_bytes;
    go(attn_bwd_q64_kernel<kBwdPolyPairs, true>, smem, std::integral_constant<int, 31>{});
  } else if (split) {
    constexpr int smem = BwdQ64Smem<false>::kBytes + 1024 + barrier_bytes;
    go(attn_bwd_q64_kernel<kBwdPolyPairs, false>, smem, std::integral_constant<int, 32>{});
  } else {
    constexpr int smem = BwdSmem<128>::kBytes + 1024 + barrier_bytes;
    if (kp == 0) go(attn_bwd_kernel<128, 0>, smem, std::integral_constant<int, 13>{});
    else if (kp == 3) go(attn_bwd_kernel<128, 3>, smem, std::integral_constant<int, 14>{});
    else if (kp == 7) go(attn_bwd_kernel<128, 7>, smem, std::integral_constant<int, 15>{});
    else go(attn_bwd_kernel<128, kBwdPolyPairs>, smem, std::integral_constant<int, 3>{});
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(err, errlen, "attention_bwd launch: %s", cudaGetErrorString(e));
    return (int)e;
  }
  if (split) {
    // dQ pass: 128-row Q / dO boxes, one CTA per (query tile, head), heaviest first
    CUtensorMap mq2, mdo2;
    if (!make_map3(&mq2, f.q, (long)f.Hq * f.hd, f.S, f.B, f.ld_q) ||
        !make_map3(&mdo2, a.dout, (long)f.Hq * f.hd, f.S, f.B, a.ld_do)) {
      snprintf(err, errlen, "attention_bwd: tensor map encode failed");
      return -1;
    }
    constexpr int smem = BwdDqSmem<128>::kBytes + 1024 + barrier_bytes;
    set_smem_once<33>(attn_bwd_dq_kernel<128, kBwdPolyPairs>, smem, device);
    const int nq = (f.S + kTile - 1) / kTile;
    attn_bwd_dq_kernel<128, kBwdPolyPairs><<<dim3(nq, f.B * f.Hq), kBwdDqThreads, smem, s>>>(
        mq2, mk, mv, mdo2, p, reinterpret_cast<__nv_bfloat16*>(a.dq), a.ld_dq);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
      snprintf(err, errlen, "attention_bwd dq pass: %s", cudaGetErrorString(e));
      return (int)e;
    }
    return 0;
  }
  const long total = rows * f.hd;
  attn_dq_convert_kernel<<<(unsigned)((total / 8 + 255) / 256), 256, 0, s>>>(
      a.dq_accum, reinterpret_cast<__nv_bfloat16*>(a.dq), a.ld_dq, f.B, f.S, f.Hq, f.hd, f.scale);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(err, errlen, "attention_bwd convert: %s", cudaGetErrorString(e));
    return (int)e;
  }
  return 0;
}

}  // namespace mt

// ============================================================================
// mt_attention_bwd_noalloc -- attention backward that allocates no memory.
//
// This entry point has no counterpart in the reference (the reference has no
// native code at all).  It is for callers that cannot call cudaMalloc: code
// running under a host framework that owns every device allocation (a fixed
// arena or memory pool that outside allocations would break), code that must
// not allocate because cudaMalloc can synchronise the device in the middle of
// its work, and plain C callers that have no caching allocator.  It runs the
// same three kernels as attention_bwd; what differs is where their scratch
// lives.  The fp32 dQ accumulator and the per-row delta = rowsum(dO * O) sit in
// one file-scope device array instead of freshly allocated buffers.  The caller
// still passes every input and output.
//
// Limits and behaviour:
//  * The array holds kNoAllocScratchFloats floats (16 MiB).  Every GPU that
//    loads this library holds it until the process exits.  A call needs
//    B*S*Hq*hd (rounded up to 64) + B*Hq*S floats; a larger problem is rejected
//    with a message and nothing is launched.
//  * The first call on a device (the device current at the call) looks up the
//    array's device address with cudaGetSymbolAddress and sets the kernels'
//    shared-memory limit for that device.  Make that first call before any
//    stream capture.
//  * Every call on a device shares the one array, which keeps the previous
//    call's contents.  The dQ accumulator is cleared at the start of each call;
//    delta is fully rewritten.  Calls that overlap on the GPU (other streams or
//    threads) race on the array: serialise them.
//  * Every pointer must be non-NULL; dout, o, q, k, v, dq, dk and dv must be
//    16-byte aligned (the kernels move them 16 bytes at a time) and lse 4-byte
//    aligned.  All checks and tensor-map encodes happen before the first launch,
//    so a rejected call queues no work.
//  * A kernel that gives up a bounded wait ORs a code into `device_status`
//    (a 4-byte device word the caller owns) or, when that is NULL, into a word
//    of this library that mt_attention_noalloc_status() returns and clears; the
//    return value only reports host-side failures.
// Returns 0 on success, otherwise non-zero with a one-line message in err.
// ============================================================================

namespace {
constexpr long kNoAllocScratchFloats = 4L << 20;
}  // namespace

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
static __device__ __align__(256) uint32_t g_noalloc_status[64];

namespace {

struct NoAllocDevice {
  float* scratch = nullptr;
  uint32_t* status = nullptr;
  bool ready = false;
};
NoAllocDevice g_noalloc_dev[64];
std::mutex g_noalloc_mu;

int noalloc_setup(int dev, char* err, int errlen) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (d.ready) return 0;
  // Host code must not use the arrays' names as device addresses: ask the
  // runtime for this device's copies.
  cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.scratch), g_noalloc_scratch);
  if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.status), g_noalloc_status);
  if (e != cudaSuccess) {
    snprintf(err, errlen, "attention_bwd_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
             cudaGetErrorString(e));
    d.scratch = nullptr;
    d.status = nullptr;
    return (int)e;
  }
  set_smem(mt::attn_bwd_kernel<64, mt::kBwdPolyPairs>, mt::BwdSmem<64>::kBytes + 1024 + 256);
  set_smem(mt::attn_bwd_kernel<128, mt::kBwdPolyPairs>, mt::BwdSmem<128>::kBytes + 1024 + 256);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(err, errlen, "attention_bwd_noalloc: set-up on device %d failed: %s", dev, cudaGetErrorString(e));
    return (int)e;
  }
  d.ready = true;
  return 0;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int mt_attention_bwd_noalloc(
    const void* dout, long ld_do, const void* q, long ld_q, const void* k, long ld_k, const void* v, long ld_v,
    const void* o, long ld_o, const float* lse, void* dq, long ld_dq, void* dk, long ld_dk, void* dv, long ld_dv,
    int B, int S, int Hq, int Hk, int hd, float scale, int causal, cudaStream_t stream, uint32_t* device_status,
    char* err, int errlen) {
  using namespace mt;
  char local_err[256];
  if (err == nullptr || errlen <= 0) {
    err = local_err;
    errlen = (int)sizeof(local_err);
  }
  err[0] = 0;
  if (B < 0 || S < 0 || Hq <= 0 || Hk <= 0) {
    snprintf(err, errlen, "attention_bwd_noalloc: bad sizes B=%d S=%d Hq=%d Hk=%d", B, S, Hq, Hk);
    return -1;
  }
  {
    const void* vec16[8] = {dout, o, q, k, v, dq, dk, dv};
    const char* names[8] = {"dout", "o", "q", "k", "v", "dq", "dk", "dv"};
    for (int i = 0; i < 8; ++i) {
      if (vec16[i] == nullptr || (reinterpret_cast<uintptr_t>(vec16[i]) & 15)) {
        snprintf(err, errlen, "attention_bwd_noalloc: %s is %s", names[i],
                 vec16[i] == nullptr ? "NULL" : "not 16-byte aligned");
        return -1;
      }
    }
    if (lse == nullptr || (reinterpret_cast<uintptr_t>(lse) & 3)) {
      snprintf(err, errlen, "attention_bwd_noalloc: lse is %s", lse == nullptr ? "NULL" : "not 4-byte aligned");
      return -1;
    }
    if (device_status != nullptr && (reinterpret_cast<uintptr_t>(device_status) & 3)) {
      snprintf(err, errlen, "attention_bwd_noalloc: device_status is not 4-byte aligned");
      return -1;
    }
  }
  AttnArgs f{};
  f.q = q;
  f.k = k;
  f.v = v;
  f.ld_q = ld_q;
  f.ld_k = ld_k;
  f.ld_v = ld_v;
  f.o = const_cast<void*>(o);
  f.ld_o = ld_o;
  f.lse = const_cast<float*>(lse);
  f.B = B;
  f.S = S;
  f.Hq = Hq;
  f.Hk = Hk;
  f.hd = hd;
  f.scale = scale;
  f.causal = causal != 0;
  if (check_args(f, err, errlen)) return -1;
  if ((ld_do | ld_dq | ld_dk | ld_dv) & 7) {
    snprintf(err, errlen, "attention_bwd_noalloc: row strides must be multiples of 8 elements");
    return -1;
  }
  if (B == 0 || S == 0) return 0;
  const long acc_floats = (long)B * S * Hq * hd;
  const long acc_pad = (acc_floats + 63) / 64 * 64;
  const long need = acc_pad + (long)B * Hq * S;
  if (need > kNoAllocScratchFloats) {
    snprintf(err, errlen,
             "attention_bwd_noalloc: problem needs %ld floats of scratch, the static buffer holds %ld "
             "(use the allocating attention_bwd for larger problems)",
             need, kNoAllocScratchFloats);
    return -3;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    snprintf(err, errlen, "attention_bwd_noalloc: no usable current device");
    return -4;
  }
  if (int rc = noalloc_setup(dev, err, errlen)) return rc;
  float* dq_accum = g_noalloc_dev[dev].scratch;
  float* delta = dq_accum + acc_pad;
  uint32_t* status = device_status ? device_status : g_noalloc_dev[dev].status;

  // Encode every tensor map first: a failed encode returns before any launch.
  CUtensorMap mq, mk, mv, mdo, mdq;
  if (!make_map3(&mq, q, (long)Hq * hd, S, B, ld_q) || !make_map3(&mk, k, (long)Hk * hd, S, B, ld_k) ||
      !make_map3(&mv, v, (long)Hk * hd, S, B, ld_v) || !make_map3(&mdo, dout, (long)Hq * hd, S, B, ld_do) ||
      !make_map3_f32(&mdq, dq_accum, (long)Hq * hd, S, B)) {
    snprintf(err, errlen, "attention_bwd_noalloc: tensor map encode failed");
    return -1;
  }
  e = cudaMemsetAsync(dq_accum, 0, acc_floats * sizeof(float), stream);
  if (e != cudaSuccess) {
    snprintf(err, errlen, "attention_bwd_noalloc: clearing scratch failed: %s", cudaGetErrorString(e));
    return (int)e;
  }
  const long rows = (long)B * S * Hq;
  attn_delta_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout), ld_do, reinterpret_cast<const __nv_bfloat16*>(o), ld_o, delta, B,
      S, Hq, hd);
  BwdParams p{};
  p.lse = lse;
  p.delta = delta;
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk);
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv);
  p.ld_dk = ld_dk;
  p.ld_dv = ld_dv;
  p.B = B;
  p.S = S;
  p.Hq = Hq;
  p.Hk = Hk;
  p.scale_log2 = scale * kLog2e;
  p.scale = scale;
  p.causal = causal ? 1 : 0;
  p.status = status;
  const dim3 grid = bwd_grid(S, B, Hk, dev);
  if (hd == 64)
    attn_bwd_kernel<64, kBwdPolyPairs><<<grid, kBwdThreads, BwdSmem<64>::kBytes + 1024 + 256, stream>>>(mq, mk, mv, mdo, mdq, p);
  else
    attn_bwd_kernel<128, kBwdPolyPairs><<<grid, kBwdThreads, BwdSmem<128>::kBytes + 1024 + 256, stream>>>(mq, mk, mv, mdo, mdq, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(err, errlen, "attention_bwd_noalloc launch: %s", cudaGetErrorString(e));
    return (int)e;
  }
  attn_dq_convert_kernel<<<(unsigned)((acc_floats / 8 + 255) / 256), 256, 0, stream>>>(
      dq_accum, reinterpret_cast<__nv_bfloat16*>(dq), ld_dq, B, S, Hq, hd, scale);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(err, errlen, "attention_bwd_noalloc convert: %s", cudaGetErrorString(e));
    return (int)e;
  }
  return 0;
}

// Reads and clears the library's own status word of the current device: the
// word that mt_attention_bwd_noalloc's kernels report a bounded-wait timeout
// into when the caller passes no device_status.  Copies four bytes each way
// (synchronously: it waits for earlier work on the device), allocates nothing.
// Returns 0 on success with the word in *out, otherwise non-zero with a message.
extern "C" __attribute__((visibility("default"))) int mt_attention_noalloc_status(uint32_t* out, char* err,
                                                                                   int errlen) {
  char local_err[256];
  if (err == nullptr || errlen <= 0) {
    err = local_err;
    errlen = (int)sizeof(local_err);
  }
  err[0] = 0;
  if (out == nullptr) {
    snprintf(err, errlen, "attention_noalloc_status: out is NULL");
    return -1;
  }
  *out = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    snprintf(err, errlen, "attention_noalloc_status: no usable current device");
    return -4;
  }
  if (int rc = noalloc_setup(dev, err, errlen)) return rc;
  uint32_t* word = g_noalloc_dev[dev].status;
  uint32_t value = 0;
  e = cudaMemcpy(&value, word, sizeof(value), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && value != 0) e = cudaMemset(word, 0, sizeof(value));
  if (e != cudaSuccess) {
    snprintf(err, errlen, "attention_noalloc_status: %s", cudaGetErrorString(e));
    return (int)e;
  }
  *out = value;
  return 0;
}

#ifdef MT_ATTN_TRACE
// Device address of the timestamp buffer of diagnostic builds.
extern "C" __attribute__((visibility("default"))) void* mt_attn_trace_buffer() {
  void* ptr = nullptr;
  cudaGetSymbolAddress(&ptr, mt::g_attn_trace);
  return ptr;
}
#endif
