// sm100.cuh -- thin inline-PTX layer for Blackwell (sm_100a) kernels.
//
// Everything the hand-written kernels of this package need from the 5th-gen
// tensor core path lives here: mbarriers with bounded waits, TMA tile loads,
// TMEM allocation, tcgen05.mma issue/commit, tcgen05.ld and the shared-memory
// matrix descriptors.  Bit layouts follow the public PTX ISA for tcgen05 (the
// UMMA smem descriptor: start>>4 in [0,14), LBO>>4 in [16,30), SBO>>4 in
// [32,46), version 1 at bit 46, swizzle mode in [61,64); the kind::f16
// instruction descriptor: D format at bit 4, A/B formats at bits 7/10, A/B
// major at bits 15/16, N>>3 at bit 17, M>>4 at bit 24).
//
// Every wait on an mbarrier is bounded by a clock budget.  When the budget runs
// out the waiting thread records an error code in a global status word and the
// kernel unwinds (see MT_WAIT_BUDGET_CYCLES); nothing in this package spins
// forever or traps.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef MT_WAIT_BUDGET_CYCLES
// ~1.5 s at 1.9 GHz.  A healthy pipeline never waits anywhere near this long.
#define MT_WAIT_BUDGET_CYCLES (3000000000ull)
#endif

namespace mt {

// Error codes written into the status word by a kernel that gave up waiting.
enum : uint32_t {
  kErrNone = 0,
  kErrWaitFull = 1u << 0,     // consumer waited too long for a TMA stage
  kErrWaitEmpty = 1u << 1,    // producer waited too long for a free stage
  kErrWaitAccum = 1u << 2,    // epilogue waited too long for the accumulator
  kErrWaitAccEmpty = 1u << 3, // MMA issuer waited too long for the epilogue
  kErrTmemAlloc = 1u << 4,    // TMEM allocation returned an unusable address
  kErrWaitPeer = 1u << 5,     // a wait on another CTA or rank ran out
  // debug builds (-DMT_DEBUG_CHECKS) only: a check failed and the access was skipped
  kErrCheckIndex = 1u << 8,    // an index read from the data (token id, target) out of range
  kErrCheckTmem = 1u << 9,     // a TMEM access past the columns the CTA allocated
  kErrCheckTma = 1u << 10,     // a TMA coordinate that is misaligned or negative where it may not be
};

// ---------------------------------------------------------------- debug checks
// With -DMT_DEBUG_CHECKS every kernel that includes this header checks the
// indices it takes from data and the TMEM / TMA addresses it forms; a failed
// check ORs a code into this translation unit's check word and skips the
// access (no trap, no fault).  The host reads and clears the words of all
// translation units with mt::read_and_clear_checks() (mt_api.h).  Release
// builds compile the checks to nothing.
void register_check_reader(uint32_t (*reader)());  // host; defined once in gemm_tcgen05.cu
#ifdef MT_DEBUG_CHECKS
static __device__ uint32_t g_check_flags;
#define MT_CHECK(cond, code)                             \
  (__builtin_expect(!(cond), 0) ? (atomicOr(&::mt::g_check_flags, (code)), false) : true)
#if !defined(__CUDA_ARCH__)
namespace {
// this translation unit's check word, read and cleared on the current device
inline uint32_t read_and_clear_unit_checks() {
  uint32_t v = 0, zero = 0;
  cudaMemcpyFromSymbol(&v, g_check_flags, sizeof(v));
  cudaMemcpyToSymbol(g_check_flags, &zero, sizeof(zero));
  return v;
}
const bool unit_checks_registered = (register_check_reader(&read_and_clear_unit_checks), true);
}  // namespace
#endif
#else
#define MT_CHECK(cond, code) true
#endif

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity.  Returns false (and records `code`
// in *status) when the clock budget runs out or another thread of the CTA has
// already flagged an abort.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          uint32_t* status, uint32_t code) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if (*abort_flag) return false;
    if ((unsigned long long)(clock64() - t0) > MT_WAIT_BUDGET_CYCLES) {
      *abort_flag = 1;
      if (status) atomicOr(status, code);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
// Order this thread's generic-proxy shared-memory writes before later async-proxy
// (TMA / tensor-core) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor load into this CTA's own shared memory only.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  if (!MT_CHECK((x & 7) == 0, kErrCheckTma)) return;  // bf16 operands: x * 2 bytes must be 16-byte aligned
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 2-D tiled load into this CTA's shared memory whose completion is counted on
// the even CTA's mbarrier of the pair (the barrier address with the pair's peer
// bit, bit 24 of the shared::cluster window, cleared).  Issued by both CTAs of
// a pair that feed one cta_group::2 MMA; each load writes only its own CTA.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  if (!MT_CHECK((x & 7) == 0, kErrCheckTma)) return;  // bf16 operands: x * 2 bytes must be 16-byte aligned
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar) & 0xFEFFFFFFu), "r"(x), "r"(y)
      : "memory");
}

// ---------------------------------------------------------------- TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------- UMMA
// Shared-memory matrix descriptor, 128-byte swizzle, tile base 1024-aligned.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;  // descriptor version for sm_100
  d |= (uint64_t)2u << 61;  // SWIZZLE_128B
  return d;
}

// Advance a shared-memory descriptor by `bytes` (a multiple of 16 inside the
// same buffer): only the 14-bit start-address field changes, and shared-memory
// addresses stay below 2^18 bytes, so the add never carries out of the field.
// Issuing loops build one descriptor per buffer up front and step it with this:
// recomputing the descriptor from a pointer per MMA costs the single issuing
// thread more cycles than a 128 x 128 x 16 MMA takes to run.
__device__ __forceinline__ uint64_t desc_add(uint64_t desc, uint32_t bytes) { return desc + (uint64_t)(bytes >> 4); }

// One lane of a converged warp (elect.sync); the tensor-core issuing roles run
// under it so the compiler sees a single-thread uniform region.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "elect.sync _|P1, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}\n"
      : "=r"(pred));
  return pred != 0;
}

// kind::f16 instruction descriptor: bf16 x bf16 -> fp32.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                          // D = F32
         | (1u << 7)                        // A = BF16
         | (1u << 10)                       // B = BF16
         | ((a_mn_major ? 1u : 0u) << 15)   // A major
         | ((b_mn_major ? 1u : 0u) << 16)   // B major
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

__device__ __forceinline__ void umma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same MMA with the A operand read from tensor memory: A is M rows (lanes) x K
// bf16 packed two per 32-bit column (element k of row m in lane m, column k/2),
// so the shared-memory port only carries B.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once every tcgen05 op issued so far by this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------- CTA pairs (cta_group::2)
// A cluster of two CTAs on neighbouring SMs shares one M=256 tensor-core tile:
// the even CTA issues the MMAs, each CTA holds half of A and half of B in its
// own shared memory and its 128 rows of the accumulator in its own TMEM.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of both CTAs; release/acquire orders shared-memory writes across the pair.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of `local`'s counterpart in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* local, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(local)), "r"(rank));
  return out;
}

// Arrive on an mbarrier of any CTA in the cluster (address from cluster_addr).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[256 x N] (+)= A[256 x 16] B[N x 16]^T across the CTA pair; issued by the even CTA only.
__device__ __forceinline__ void umma_bf16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier (shared::cluster address, either CTA of the pair) once
// every cta_group::2 tcgen05 operation issued so far by this thread completes.
__device__ __forceinline__ void umma_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
               : "memory");
}

// 32 lanes x 32 consecutive fp32 columns: thread i of the warp gets lane (base+i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, float* v) {
  if (!MT_CHECK((taddr & 0xFFFFu) + 32u <= 512u, kErrCheckTmem)) return;
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}


// 32 lanes x 64 consecutive fp32 columns, then wait: thread i gets lane (base+i).
__device__ __forceinline__ void tmem_ld_32x32b_x64(uint32_t taddr, float* v) {
  if (!MT_CHECK((taddr & 0xFFFFu) + 64u <= 512u, kErrCheckTmem)) return;
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr) : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 128 consecutive fp32 columns, then wait: thread i gets lane (base+i).
__device__ __forceinline__ void tmem_ld_32x32b_x128(uint32_t taddr, float* v) {
  if (!MT_CHECK((taddr & 0xFFFFu) + 128u <= 512u, kErrCheckTmem)) return;
  uint32_t r[128];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
      : "r"(taddr) : "memory");
#pragma unroll
  for (int i = 0; i < 128; ++i) v[i] = __uint_as_float(r[i]);
}

// 2^x on the special-function unit (PTX ex2.approx.ftz.f32).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 32 lanes x 32 consecutive fp32 columns store (thread i writes lane base+i).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const float* v) {
  if (!MT_CHECK((taddr & 0xFFFFu) + 32u <= 512u, kErrCheckTmem)) return;
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 16 consecutive 32-bit columns, no wait (pair with tmem_wait_st).
__device__ __forceinline__ void tmem_st_32x32b_x16_nowait(uint32_t taddr, const uint32_t* r) {
  if (!MT_CHECK((taddr & 0xFFFFu) + 16u <= 512u, kErrCheckTmem)) return;
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- misc
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Two fp32 values rounded to bf16 (nearest, ties away from zero) and packed,
// with integer adds and one byte permute: no conversion instruction, so the
// special-function pipe stays free for the exponentials of the softmax.
// (Inputs are finite; a value that rounds past the largest bf16 becomes inf.)
__device__ __forceinline__ uint32_t pack_bf16x2_int(float lo, float hi) {
  const uint32_t a = __float_as_uint(lo) + 0x8000u;
  const uint32_t b = __float_as_uint(hi) + 0x8000u;
  return __byte_perm(a, b, 0x7632);  // bytes 2,3 of a (low half), bytes 2,3 of b (high half)
}

// Packed fp32 pairs: sm_100's f32x2 instructions do two fp32 operations per
// issue slot on a 64-bit register pair.
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t sub_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x for two values on the FMA and integer pipes instead of the special-function
// unit, which issues only 16 exponentials per SM per clock; softmax kernels send a
// share of their exponentials here so both pipes work at once.
//   x = j + f, j = rint(x) (adding 1.5 * 2^23 rounds to an integer), f in [-1/2, 1/2]
//   2^f ~ c0 + f (c1 + f (c2 + f c3)): a cubic fitted to 2^f on [-1/2, 1/2] for the
//   least maximum relative error (iteratively reweighted least squares on Chebyshev
//   nodes): 7.5e-5, far below bf16's half-ulp of 2^-9;
//   2^j enters by adding j to the exponent field: bits(x + 1.5 * 2^23) = bits(1.5 * 2^23) + j,
//   and bits(1.5 * 2^23) << 23 is 0 modulo 2^32.
// Valid for x <= 127.  x is clamped to >= -126 so the exponent cannot underflow:
// 2^-126 and below come out as about 1e-38 instead of 0 (callers that need exact
// zeros, e.g. masked entries, use ex2_approx there).
__device__ __forceinline__ uint64_t ex2_poly_x2(uint64_t x) {
  constexpr float kRound = 12582912.0f;
  float x0, x1;
  f2unpack(x, x0, x1);
  const uint64_t xc = f2pack(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
  const uint64_t rnd = f2pack(kRound, kRound);
  const uint64_t t = add_f32x2(xc, rnd);
  const uint64_t f = sub_f32x2(xc, sub_f32x2(t, rnd));
  uint64_t q = fma_f32x2(f, f2pack(0.055171653628349304f, 0.055171653628349304f),
                         f2pack(0.2426111251115799f, 0.2426111251115799f));
  q = fma_f32x2(q, f, f2pack(0.6932609677314758f, 0.6932609677314758f));
  q = fma_f32x2(q, f, f2pack(0.9999280571937561f, 0.9999280571937561f));
  uint32_t t0, t1, q0, q1;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(t0), "=r"(t1) : "l"(t));
  asm("mov.b64 {%0, %1}, %2;" : "=r"(q0), "=r"(q1) : "l"(q));
  q0 += t0 << 23;
  q1 += t1 << 23;
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(q0), "r"(q1));
  return r;
}

// Which of the 16 column pairs of a 32-column softmax chunk take ex2_poly_x2:
// K of 16, spread evenly (pair q when floor((q + 1) K / 16) > floor(q K / 16)).
template <int K>
__device__ __forceinline__ constexpr bool poly_pair(int q) {
  return ((q + 1) * K) / 16 > (q * K) / 16;
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t u) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(v);
}

// erf(z) by the rational approximation of Abramowitz & Stegun, Handbook of
// Mathematical Functions, formula 7.1.26 (|error| <= 1.5e-7 for all z):
//   erf(z) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2),  t = 1 / (1 + p |z|)
// with the handbook's constants p, a1..a5; odd symmetry for z < 0.  exp(-z^2) is
// returned too: the GELU gradient reuses it as the Gaussian density.
__device__ __forceinline__ float erf_as7126(float z, float* gauss) {
  const float a = fabsf(z);
  const float t = __fdividef(1.0f, fmaf(0.3275911f, a, 1.0f));
  const float e = ex2_approx(-(a * a) * 1.4426950408889634f);
  float poly = fmaf(t, 1.061405429f, -1.453152027f);
  poly = fmaf(t, poly, 1.421413741f);
  poly = fmaf(t, poly, -0.284496736f);
  poly = fmaf(t, poly, 0.254829592f);
  *gauss = e;
  return copysignf(fmaf(-t * poly, e, 1.0f), z);
}

// GELU (exact form, x * Phi(x)) and its derivative Phi(x) + x phi(x).
__device__ __forceinline__ float gelu_erf(float x) {
  float g;
  return 0.5f * x * (1.0f + erf_as7126(x * 0.70710678118654752f, &g));
}

__device__ __forceinline__ float gelu_erf_grad(float x) {
  float g;  // exp(-x^2 / 2)
  const float cdf = 0.5f * (1.0f + erf_as7126(x * 0.70710678118654752f, &g));
  return cdf + x * (0.39894228040143268f * g);
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

}  // namespace mt
