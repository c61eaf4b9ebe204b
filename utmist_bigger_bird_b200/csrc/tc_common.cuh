// tcgen05 / TMA / mbarrier building blocks shared by the sm_100a kernels (attention and routing).
//
// Conventions: 128-row x 128-column 16-bit tiles (TILE bytes) stored as two 64-column halves
// (HALF bytes each, one 128-byte swizzle span per row); K-major operands use the 128B-swizzled
// layout TMA writes. Every mbarrier wait is bounded: on expiry the waiter raises the CTA's abort
// flag and records `code` in this translation unit's fault word.
#pragma once
#include <cudaTypedefs.h>

#include <atomic>

#include "bb_common.cuh"

namespace bb {
namespace tc {

constexpr uint32_t TILE = 32768u;  // 128 rows x 128 columns x 2 bytes
constexpr uint32_t HALF = 16384u;  // 128 rows x 64 columns (one 128-byte swizzle span per row)

// Fault word of the kernels in the including translation unit (0 = no fault): the code of the
// first bounded wait that gave up. Read and cleared by that unit's host side.
static __device__ int g_tc_fault = 0;
// Serial number of the latest launch of this unit in which a CTA gave up a wait (0 = none). The
// other CTAs of that launch read it while they spin and leave at once: without it every CTA of a
// grid would wait out its own limit, and a launch of many waves would take waves x the limit.
static __device__ unsigned int g_tc_abort = 0;
// Limit of one bounded wait in nanoseconds (bb_set_wait_limit_ns; 2 s by default).
static __device__ unsigned long long g_tc_wait_ns = 2000000000ull;

// The abort state a bounded wait consults: the CTA's shared-memory abort flag and the launch's
// serial number (0: the launch does not take part in cross-CTA aborts).
struct Abort {
  volatile uint32_t* flag;
  uint32_t serial;
};

// ----------------------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Limit of the drain waits on the way out (fixed: they wait only for copies and MMAs already
// issued, which complete on their own).
constexpr uint64_t DRAIN_LIMIT_NS = 2000000000ull;

// Waits for the phase of `parity`: false if another role of this CTA, or another CTA of this
// launch, aborted, or if the wait limit passed (then it aborts: flag, fault code, launch serial).
// Fully inline (a call here costs the hand-offs on the critical path measurably): one
// non-blocking test for the common already-completed case, then a try_wait spin that looks at
// the abort state and the clock every 64 polls.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, Abort ab, int code) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  if (ok) return true;
  // The global words (abort serial, limit) are read only on the every-64-polls check: a load left
  // in flight when the wait succeeds would stall the next write of its register on the hand-off
  // path between the warps.
  const uint64_t t0 = gtimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try(bar, parity)) return true;
    if ((it & 63) == 0) {
      if (*ab.flag) return false;
      if (ab.serial != 0 && *(volatile unsigned int*)&g_tc_abort == ab.serial) {
        *ab.flag = 1;
        return false;
      }
      if (gtimer() - t0 > *(volatile unsigned long long*)&g_tc_wait_ns) {
        *ab.flag = 1;
        atomicCAS(&g_tc_fault, 0, code);  // the first wait that gave up keeps its code
        if (ab.serial != 0) atomicExch(&g_tc_abort, ab.serial);
        return false;
      }
    }
  }
}
// mbar_wait made warp-uniform (false if any lane gave up): every lane polls, and the warp stays
// converged for the elect.sync issue or the warp-wide (.sync.aligned) TMEM accesses that follow,
// and leaves together on an abort.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, Abort ab, int code) {
  const bool ok = mbar_wait(bar, parity, ab, code);
  return __all_sync(0xffffffffu, ok);
}
// Bounded wait used while draining on the way out (ignores the abort flag).
static __device__ __noinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = gtimer();
  while (!mbar_try(bar, parity))
    if (gtimer() - t0 > DRAIN_LIMIT_NS) return;
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

// Issue-side wrappers for a converged warp: all 32 lanes execute the block, elect.sync picks the
// one lane that issues. Measured on this kernel, an elected issue keeps the tensor pipe fed
// noticeably better than the same instructions predicated on a lane-index register.
__device__ __forceinline__ void mbar_expect_tx_one(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n @e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n}\n"
               ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive_one(uint32_t bar) {
  asm volatile("{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n @e mbarrier.arrive.shared::cta.b64 _, [%0];\n}\n"
               ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tma_load_3d_one(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                                uint32_t bar) {
  asm volatile(
      "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
      " @e cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];\n}\n"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05): start >> 4 at [0,14), LBO >> 4 at [16,30), SBO >> 4
// at [32,46), fixed 0b01 at [46,48), swizzle mode at [61,64) (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// K-major, 128B-swizzled: 8-row core groups 1024 bytes apart; LBO unused.
__device__ __forceinline__ uint64_t desc_k(uint32_t saddr) { return sdesc(saddr, 16, 1024); }
// MN-major, 128B-swizzled: 64-element column blocks 16 KB apart (LBO), 8-row groups 1024 bytes (SBO).
__device__ __forceinline__ uint64_t desc_mn(uint32_t saddr) { return sdesc(saddr, HALF, 1024); }

// Instruction descriptor, kind::f16: D f32 (bit 4), A/B type at [7,10)/[10,13) (0 f16, 1 bf16),
// B major at bit 16 (1 = MN), N >> 3 at [17,23), M >> 4 at [24,29).
template <typename T> __host__ __device__ constexpr uint32_t ab_fmt();
template <> __host__ __device__ constexpr uint32_t ab_fmt<__nv_bfloat16>() { return 1u; }
template <> __host__ __device__ constexpr uint32_t ab_fmt<__half>() { return 0u; }
template <typename T> __host__ __device__ constexpr uint32_t idesc(bool b_mn, int n = 128, int m = 128) {
  return (1u << 4) | (ab_fmt<T>() << 7) | (ab_fmt<T>() << 10) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_commit_one(uint32_t bar) {
  asm volatile("{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
               " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n"
               ::"r"(bar) : "memory");
}

// A whole 128x128x128 GEMM (8 K-steps of 16) in one asm block, issued by one elected lane of a
// converged warp: the predicates are set once and every descriptor is formed before the first
// MMA, so the eight tcgen05.mma issue back to back.
// The issuing warp shares its SM sub-partition with two busy softmax warps; with one small asm
// block per step the instructions between steps lose issue slots and the tensor pipe drains.
// Both operands K-major SW128: a K-step advances the start address by 32 B (+2 in descriptor
// units) inside the 128 B row, and after four steps moves to the operand's second 64-column half
// (+1024 = 16 KB for a 128-row tile).
template <int AH = 1024, int BH = 1024>
__device__ __forceinline__ void gemm_ss8(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  // AH / BH: descriptor offset (16-byte units) of the operand's second 64-column half.
  asm volatile(
      "{\n .reg .pred q, p, t;\n .reg .b64 a1, a2, a3, a4, a5, a6, a7, b1, b2, b3, b4, b5, b6, b7;\n"
      " elect.sync _|q, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n setp.eq.b32 t, %4, %4;\n"
      " add.s64 a1, %1, 2;\n add.s64 a2, %1, 4;\n add.s64 a3, %1, 6;\n add.s64 a4, %1, %5;\n"
      " add.s64 a5, %1, %6;\n add.s64 a6, %1, %7;\n add.s64 a7, %1, %8;\n"
      " add.s64 b1, %2, 2;\n add.s64 b2, %2, 4;\n add.s64 b3, %2, 6;\n add.s64 b4, %2, %9;\n"
      " add.s64 b5, %2, %10;\n add.s64 b6, %2, %11;\n add.s64 b7, %2, %12;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], a2, b2, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], a3, b3, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], a4, b4, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], a5, b5, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], a6, b6, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], a7, b7, %3, t;\n}\n"
      ::"r"(d), "l"(a), "l"(b), "r"(id), "r"(acc), "n"(AH), "n"(AH + 2), "n"(AH + 4), "n"(AH + 6), "n"(BH),
      "n"(BH + 2), "n"(BH + 4), "n"(BH + 6));
}
// O += P V: P (A) from TMEM, 8 columns (16 packed keys) per K-step; V (B) MN-major SW128, 16 key
// rows = 2048 B (+128 in descriptor units) per K-step.
__device__ __forceinline__ void gemm_ts8(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred q, p, t;\n .reg .b32 t1, t2, t3, t4, t5, t6, t7;\n .reg .b64 b1, b2, b3, b4, b5, b6, b7;\n"
      " elect.sync _|q, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n setp.eq.b32 t, %4, %4;\n"
      " add.u32 t1, %1, 8;\n add.u32 t2, %1, 16;\n add.u32 t3, %1, 24;\n add.u32 t4, %1, 32;\n"
      " add.u32 t5, %1, 40;\n add.u32 t6, %1, 48;\n add.u32 t7, %1, 56;\n"
      " add.s64 b1, %2, 128;\n add.s64 b2, %2, 256;\n add.s64 b3, %2, 384;\n add.s64 b4, %2, 512;\n"
      " add.s64 b5, %2, 640;\n add.s64 b6, %2, 768;\n add.s64 b7, %2, 896;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], [t1], b1, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], [t2], b2, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], [t3], b3, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], [t4], b4, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], [t5], b5, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], [t6], b6, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], [t7], b7, %3, t;\n}\n"
      ::"r"(d), "r"(a_tmem), "l"(b), "r"(id), "r"(acc));
}
// Half of the P.V GEMM: 4 K-steps (64 keys) starting at P column a_tmem and V descriptor b.
__device__ __forceinline__ void gemm_ts4(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred q, p, t;\n .reg .b32 t1, t2, t3;\n .reg .b64 b1, b2, b3;\n"
      " elect.sync _|q, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n setp.eq.b32 t, %4, %4;\n"
      " add.u32 t1, %1, 8;\n add.u32 t2, %1, 16;\n add.u32 t3, %1, 24;\n"
      " add.s64 b1, %2, 128;\n add.s64 b2, %2, 256;\n add.s64 b3, %2, 384;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], [t1], b1, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], [t2], b2, %3, t;\n"
      " @q tcgen05.mma.cta_group::1.kind::f16 [%0], [t3], b3, %3, t;\n}\n"
      ::"r"(d), "r"(a_tmem), "l"(b), "r"(id), "r"(acc));
}

// 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread (load and wait together,
// so no use of the registers can be scheduled before the data has arrived).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n"
      ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
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
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

#define BB_R8(b) "=r"(r[b]), "=r"(r[b + 1]), "=r"(r[b + 2]), "=r"(r[b + 3]), "=r"(r[b + 4]), "=r"(r[b + 5]), \
                 "=r"(r[b + 6]), "=r"(r[b + 7])
#define BB_W8(b) "r"(r[b]), "r"(r[b + 1]), "r"(r[b + 2]), "r"(r[b + 3]), "r"(r[b + 4]), "r"(r[b + 5]), \
                 "r"(r[b + 6]), "r"(r[b + 7])

// One row of a 128-column S tile: a single x128 load and its wait in one asm statement.
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float* v) {
  uint32_t r[128];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,"
      "%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,"
      "%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,"
      "%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,%96,%97,%98,%99,%100,"
      "%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,"
      "%121,%122,%123,%124,%125,%126,%127}, [%128];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : BB_R8(0), BB_R8(8), BB_R8(16), BB_R8(24), BB_R8(32), BB_R8(40), BB_R8(48), BB_R8(56), BB_R8(64),
        BB_R8(72), BB_R8(80), BB_R8(88), BB_R8(96), BB_R8(104), BB_R8(112), BB_R8(120)
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 128; ++i) v[i] = __uint_as_float(r[i]);
}
// Half a row of S (64 columns): one x64 load and its wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,"
      "%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,"
      "%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : BB_R8(0), BB_R8(8), BB_R8(16), BB_R8(24), BB_R8(32), BB_R8(40), BB_R8(48), BB_R8(56)
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
// 64 packed columns (P of one row) in one store.
__device__ __forceinline__ void tmem_st64(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {"
      "%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,"
      "%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,"
      "%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64};\n"
      ::"r"(taddr), BB_W8(0), BB_W8(8), BB_W8(16), BB_W8(24), BB_W8(32), BB_W8(40), BB_W8(48), BB_W8(56)
      : "memory");
}
#undef BB_R8
#undef BB_W8

__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ----------------------------------------------------------------------------- host side
// Per-unit control of the wait state above (each translation unit that includes this header has
// its own copies; these helpers act on the including unit's symbols, on the current device).
static inline int unit_set_wait_limit(unsigned long long ns) {
  return cudaMemcpyToSymbol(g_tc_wait_ns, &ns, sizeof(ns)) == cudaSuccess ? 0 : -1;
}
// Next launch serial of the including unit (never 0).
static inline uint32_t unit_next_serial() {
  static std::atomic<uint32_t> serial{0};
  uint32_t s = serial.fetch_add(1, std::memory_order_relaxed) + 1;
  if (s == 0) s = serial.fetch_add(1, std::memory_order_relaxed) + 1;
  return s;
}
// cuTensorMapEncodeTiled through the runtime's driver entry point (nullptr if unavailable).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();
// 3-D TMA map over a [heads][rows][128] 16-bit view with element strides (s_head, s_row), box
// {64, 128 rows, 1 head}, 128-byte swizzle; the two outer dimensions are ordered by stride
// (*swap = 1 when the head stride is the smaller one).
int make_map(CUtensorMap* m, int* swap, const void* base, int dtype, int64_t heads, int64_t rows,
             int64_t s_head, int64_t s_row);

}  // namespace tc
}  // namespace bb
