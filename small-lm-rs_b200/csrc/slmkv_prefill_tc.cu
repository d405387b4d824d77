// Causal GQA prefill attention over a bf16 paged cache on the 5th-generation
// tensor cores (tcgen05): the batched prompt path of
// ProjectedQkv::{scaled_causal_scores, causal_probabilities, attend_values}
// (rust/engine/src/attention.rs:195-399) with the cache of
// forward_prefill_with_cache (attention.rs:835-870).
//
// A CTA covers 256 query rows of one (sequence, KV head) as two 128-row
// query tiles (A, B); a query tile is the G query heads of the group times
// 128/G consecutive new tokens (row r = token r/G, head r%G), so every K/V
// tile is shared by the whole group. Per 128-token K/V tile and query tile:
//   S = Q K^T        tcgen05.mma kind::f16, M=128 N=128, f32 in TMEM; Q
//                    rounded to bf16 after RoPE and scaling
//   softmax          one warpgroup per query tile, one row per thread (TMEM
//                    lane = row), exp2 domain, causal mask; the running max
//                    moves only when a row's max grows by more than 2^8, then
//                    O is rescaled in TMEM
//   O += P V         M=128 N=64, P (bf16) from TMEM, V as an MN-major
//                    operand from shared memory, O in TMEM
// Q, K and V tiles are 128-byte-swizzled: K/V blocks arrive by TMA (16 rows
// per block, block-table lookups), Q is written by the threads in the same
// layout.
#include <cfloat>
#include <cstdint>

#include "slmkv_internal.h"

namespace slmkv {
namespace {

constexpr int kTileM = 128;    // query rows per CTA
constexpr int kTileN = 128;    // K/V tokens per tile (8 blocks)
constexpr int kTileBytes = kTileN * kHeadDim * 2;  // 16 KiB: 128 rows of 128 B
constexpr float kScaleLog2Tc = 0.125f * 1.4426950408889634f;
constexpr unsigned long long kWaitNs = 1000000000ull;  // 1 s
constexpr int kWaitSpinsMax = 1 << 26;

__device__ __forceinline__ uint32_t su32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: true when the phase completed, false after ~1 s.
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
  if (bar_try(bar, parity)) return true;
  const unsigned long long t0 = gtimer();
  for (int i = 0; i < kWaitSpinsMax; ++i) {
    if (bar_try(bar, parity)) return true;
    if ((i & 255) == 255 && gtimer() - t0 > kWaitNs) return false;
  }
  return false;
}
__device__ __forceinline__ void tma_rows(uint32_t dst, const CUtensorMap* map, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(bar)
      : "memory");
}
// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 layout: start
// address, leading / stride byte offsets in 16-byte units, version 1).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo16, uint32_t sbo16) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>(lbo16 & 0x3FFFu) << 16) |
         (static_cast<uint64_t>(sbo16 & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: f32 accumulate, bf16 A and B, A K-major.
constexpr uint32_t idesc(int m, int n, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t id,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(id), "r"(accumulate)
      : "memory");
}
// The same with A read from TMEM (M rows in lanes, K along columns, two bf16
// per 32-bit column, the lower k in the low half).
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t id,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(id), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
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
}
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]),
      "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]),
      "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Three-input max (sm_100): fewer instructions for a row's max.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// Two f32 lanes in one 64-bit register, for the packed f32x2 arithmetic.
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {  // two IEEE adds, rounded to nearest
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {  // a * b + c, twice
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// MMA operands (Q, P) to bf16, round to nearest even, one instruction per pair.
__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// Byte offset of 16-byte unit u of row r in a 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t swz(int r, int u) {
  return static_cast<uint32_t>(((r >> 3) << 10) + ((r & 7) << 7) + (((u ^ r) & 7) << 4));
}

// A CTA is QT softmax warpgroups and a producer warpgroup. Softmax warpgroup
// w owns a 128-row query tile (w = 0: the CTA's first 128/G tokens, w = 1: the
// next 128/G); in the producer warpgroup, the first warp loads K/V tiles (3
// stages each), the second issues the S = Q K^T products and the third the
// O += P V products. TMEM holds S, O and P of the CTA's query tiles; with
// QT = 1 two CTAs share an SM, with QT = 2 the two tiles of one CTA do, so
// either way the tensor cores compute one tile's scores while another
// tile's softmax runs. Every handoff is an mbarrier:
//   k_full/v_full[s]  copies landed (TMA transaction bytes)   loader -> MMA
//   k_free/v_free[s]  the MMAs reading the stage are done     MMA -> loader
//   q_full[w]         Q tile w written (4 warp arrivals)      softmax -> S
//   s_full[w]         S_w of the next K tile is in TMEM       S -> softmax
//   s_free[w]         S_w read out of TMEM (4 arrivals)       softmax -> S
//   p_full[w]         P_w in TMEM, O_w rescaled               softmax -> PV
//   o_done[w]         P_w V done: P_w and O_w free            PV -> softmax
// Each completes once per K/V tile in order, so its phase parity is the
// tile index's low bit. The two issuers touch disjoint TMEM columns, and each
// commits only its own MMAs. Registers are rebalanced with setmaxnreg: the
// softmax warpgroups rise (a 128-score row stays in registers), the
// producer warpgroup drops, within the registers the CTA is launched with
// (checked on the host before launch).
// A wait that runs out (1 s) sets the CTA's abort flag, which ends every
// other wait at once; the loader then waits (bounded) for its own copies and
// each issuer for its own MMAs before TMEM is released.
constexpr int kWsStages = 3;
constexpr int kPrefillQT = 1;  // query tiles per CTA (1: two CTAs per SM)
// Launch shape for QT query tiles per CTA (128 threads each) plus the
// producer warpgroup. QT = 2: one CTA per SM (384 threads at 168 registers,
// 512 TMEM columns). QT = 1: two CTAs per SM (256 threads at 128 registers,
// 256 TMEM columns, 112 KiB of shared memory each), so one CTA's start and
// end overlap the other's steady state.
// TMEM columns: S_w [128w, +128), O_w [128QT + 64w, +64), P_w [192QT + 64w,
// +64) (P: 128 bf16 a row, two a column).
template <int QT>
struct WsCfg {
  static constexpr int kThreads = 128 * (QT + 1);
  static constexpr int kCtasPerSm = QT == 1 ? 2 : 1;
  static constexpr int kTmemCols = 256 * QT;
  static constexpr int kOCol = 128 * QT;
  static constexpr int kPCol = 192 * QT;
  static constexpr int kRegsLaunch = (65536 / (kThreads * kCtasPerSm)) / 8 * 8;
  static constexpr int kRegsSoftmax = QT == 2 ? 224 : 216;
  static constexpr int kRegsProducer = QT == 2 ? 56 : 40;
  static_assert(128 * (QT * kRegsSoftmax + kRegsProducer) <= kThreads * kRegsLaunch,
                "the setmaxnreg split must fit the registers the CTA is launched with");
  static constexpr int kOffQ = 0;                                    // Q_w
  static constexpr int kOffK = kOffQ + QT * kTileBytes;                // kWsStages buffers
  static constexpr int kOffV = kOffK + kWsStages * kTileBytes;         // kWsStages buffers
  static constexpr int kOffBar = kOffV + kWsStages * kTileBytes;
};
enum : int {
  kBarKFull = 0,
  kBarVFull = kBarKFull + kWsStages,
  kBarKFree = kBarVFull + kWsStages,
  kBarVFree = kBarKFree + kWsStages,
  kBarQFull = kBarVFree + kWsStages,
  kBarSFull = kBarQFull + 2,
  kBarSFree = kBarSFull + 2,
  kBarPFull = kBarSFree + 2,
  kBarODone = kBarPFull + 2,
  kBarDrain = kBarODone + 2,  // one per MMA-issuing warp
  kWsBars = kBarDrain + 2
};
template <int QT>
constexpr int ws_off_misc() {  // TMEM base, abort flag
  return WsCfg<QT>::kOffBar + 8 * kWsBars;
}
template <int QT>
constexpr int ws_smem() {
  return ws_off_misc<QT>() + 16;
}

__device__ __forceinline__ void bar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ uint32_t ld_volatile_shared(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.volatile.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_volatile_shared(uint32_t addr, uint32_t v) {
  asm volatile("st.volatile.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
// The value, hidden from the optimizer: addresses derived from it inside a
// loop are recomputed there instead of being kept in registers across the
// loop (the producer warps run with few registers).
__device__ __forceinline__ uint32_t opaque(uint32_t x) {
  asm volatile("" : "+r"(x));
  return x;
}
// Bounded wait that also gives up as soon as another role raised the abort
// flag (a shared-memory word at abort_addr).
__device__ __forceinline__ bool bar_wait_ab(uint32_t bar, uint32_t parity, uint32_t abort_addr) {
  if (bar_try(bar, parity)) return true;
  const unsigned long long t0 = gtimer();
  for (int i = 0; i < kWaitSpinsMax; ++i) {
    if (bar_try(bar, parity)) return true;
    if (ld_volatile_shared(abort_addr)) return false;
    if ((i & 255) == 255 && gtimer() - t0 > kWaitNs) return false;
  }
  return false;
}

// The CTA's share of the launch, derived from the block indices. Each role
// derives it again after its setmaxnreg (the special-register reads are
// volatile and the sequence entry is loaded again), so that nothing but the
// shared-memory base stays live across the register reallocation, which
// would otherwise move such values through local memory.
struct CtaWork {
  SeqEntry se;
  int h, q0;
  int nq0, nq1;  // query tile w: tokens [q0 + w*TQ, +nq_w)
  int nt0, nt1;  // ... attends K/V tiles [0, nt_w)
  int n_kv;      // keys the CTA reads
  int n_load;    // K/V tiles the CTA loads: max(nt0, nt1) = (n_kv + 127) / 128
};
__device__ __forceinline__ int thread_index() {
  uint32_t t;
  asm volatile("mov.u32 %0, %%tid.x;" : "=r"(t));
  return static_cast<int>(t);
}
template <int G, int QT>
__device__ __forceinline__ CtaWork cta_work(const PrefillLaunch& p) {
  // Grid (KV head, sequence, query-tile rank): blocks start in that linear
  // order, so the query tiles furthest into the prompts (the most K/V tiles)
  // of every sequence and head start first and the short ones fill the tail.
  uint32_t bx, by, bz, nbz;
  asm volatile("mov.u32 %0, %%ctaid.x;" : "=r"(bx));
  asm volatile("mov.u32 %0, %%ctaid.y;" : "=r"(by));
  asm volatile("mov.u32 %0, %%ctaid.z;" : "=r"(bz));
  asm volatile("mov.u32 %0, %%nctaid.z;" : "=r"(nbz));
  constexpr int TQ = kTileM / G;
  CtaWork c;
  c.se = p.seqs[by];
  c.h = static_cast<int>(bx);
  c.q0 = (static_cast<int>(nbz) - 1 - static_cast<int>(bz)) * QT * TQ;
  c.nq0 = min(TQ, c.se.count - c.q0);
  c.nq1 = QT == 2 ? max(0, min(TQ, c.se.count - c.q0 - TQ)) : 0;
  c.nt0 = (c.se.base + c.q0 + c.nq0 - 1) / kTileN + 1;
  c.nt1 = c.nq1 > 0 ? (c.se.base + c.q0 + TQ + c.nq1 - 1) / kTileN + 1 : 0;
  c.n_kv = c.se.base + c.q0 + c.nq0 + c.nq1;
  c.n_load = max(c.nt0, c.nt1);
  return c;
}

template <int G, int QT>
__global__ void __launch_bounds__(WsCfg<QT>::kThreads, WsCfg<QT>::kCtasPerSm)
    prefill_ws_kernel(const __grid_constant__ PrefillLaunch p) {
  SLMKV_TL(kTlPrefillTc);
  using Cfg = WsCfg<QT>;
  static_assert(ws_smem<QT>() <= 227 * 1024 &&
                    Cfg::kCtasPerSm * (ws_smem<QT>() + 1024) <= 228 * 1024,
                "the CTAs of an SM must fit its shared memory");
  constexpr int kLoadWarp = 4 * QT, kSWarp = 4 * QT + 1, kPvWarp = 4 * QT + 2;
  extern __shared__ __align__(1024) uint8_t sm[];
  const uint32_t sbase = su32(sm);
  if (sbase & 1023u) {  // uniform over the CTA: report instead of misreading tiles
    if (threadIdx.x == 0) atomicOr(p.g.error, kErrLayout);
    return;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int TQ = kTileM / G;  // new tokens per query tile
  {
    const CtaWork c = cta_work<G, QT>(p);
    if (c.q0 >= c.se.count) return;  // uniform over the CTA
  }

  auto bar = [&](int i) { return sbase + Cfg::kOffBar + 8u * static_cast<uint32_t>(i); };
  const uint32_t abort_off = ws_off_misc<QT>() + 4;  // the abort flag's shared-memory offset
  if (tid == 0) {
    for (int s = 0; s < kWsStages; ++s) {
      bar_init(bar(kBarKFull + s), 1);
      bar_init(bar(kBarVFull + s), 1);
      bar_init(bar(kBarKFree + s), 1);
      bar_init(bar(kBarVFree + s), 1);
    }
    for (int w = 0; w < 2; ++w) {
      bar_init(bar(kBarQFull + w), 4);
      bar_init(bar(kBarSFull + w), 1);
      bar_init(bar(kBarSFree + w), 4);
      bar_init(bar(kBarPFull + w), 4);
      bar_init(bar(kBarODone + w), 1);
    }
    bar_init(bar(kBarDrain + 0), 1);
    bar_init(bar(kBarDrain + 1), 1);
    st_volatile_shared(sbase + abort_off, 0u);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kSWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     sbase + ws_off_misc<QT>()),
                 "r"(Cfg::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // One lane of a warp reports a failed (warp-uniform) wait.
  auto raise_abort = [&]() {
    if (lane == 0) {
      st_volatile_shared(sbase + abort_off, 1u);
      atomicOr(p.g.error, kErrTimeout);
    }
  };
  auto wait_warp = [&](uint32_t b, uint32_t parity) {
    const bool ok = bar_wait_ab(b, parity, sbase + abort_off);
    return __all_sync(0xffffffffu, ok);
  };

  if (warp < 4 * QT) {
    // ================= softmax warpgroups =================
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(Cfg::kRegsSoftmax) : "memory");
    const CtaWork cw = cta_work<G, QT>(p);
    const SeqEntry se = cw.se;
    const int h = cw.h, q0 = cw.q0, nq0 = cw.nq0, nq1 = cw.nq1, nt0 = cw.nt0, nt1 = cw.nt1;
    const int Hq = p.g.q_heads;
    const uint32_t tmem = ld_volatile_shared(sbase + ws_off_misc<QT>());
    const int w = warp >> 2;
    const int r = tid & 127;  // this thread's row = TMEM lane
    const int qw0 = q0 + w * TQ, nqw = w ? nq1 : nq0, ntw = w ? nt1 : nt0;
    const int tq = r / G, gq = r % G;
    const bool live = tq < nqw;
    const int qpos = se.base + qw0 + tq;
    const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t s_col = static_cast<uint32_t>(w * kTileN), o_col = Cfg::kOCol + w * kHeadDim,
                   p_col = Cfg::kPCol + w * (kTileN / 2);
    if (ntw > 0) {
      // Q rows: RoPE at the token's position, scaled into the exp2 domain,
      // bf16; rows past the tile's tokens are zero. A warp writes its 32 TMEM
      // rows one row per step: lane l holds elements 2l, 2l+1 (one RoPE pair),
      // so each row is one coalesced 256-byte load (and one of the RoPE
      // table), and the lanes' 4-byte results fill the row's swizzled line.
      uint8_t* qt = sm + Cfg::kOffQ + w * kTileBytes;
      const int r0 = (warp & 3) * 32;
      float2 xv[32], cv[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {  // all loads first
        const int t = (r0 + i) / G, g = (r0 + i) % G;
        const bool lv = t < nqw;
        const size_t row = static_cast<size_t>(se.row_offset + qw0 + t) * Hq + h * G + g;
        xv[i] = lv ? reinterpret_cast<const float2*>(p.q + row * kHeadDim)[lane] : make_float2(0.f, 0.f);
        cv[i] = lv && p.rotate
                    ? p.g.rope[static_cast<size_t>(se.base + qw0 + t) * (kHeadDim / 2) + lane]
                    : make_float2(1.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float2 x = xv[i];
        if (p.rotate) {
          const float2 c = cv[i];
          x = make_float2(__fsub_rn(__fmul_rn(x.x, c.x), __fmul_rn(x.y, c.y)),
                          __fadd_rn(__fmul_rn(x.x, c.y), __fmul_rn(x.y, c.x)));
        }
        *reinterpret_cast<uint32_t*>(qt + swz(r0 + i, lane >> 2) + (lane & 3) * 4) =
            bf16x2(x.x * kScaleLog2Tc, x.y * kScaleLog2Tc);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) bar_arrive(bar(kBarQFull + w));
    }
    // fin2: +0 in both halves while every score of the row (masked ones are
    // finite) has been finite; a NaN from the first non-finite one on.
    float m_used = -INFINITY, l_sum = 0.f;
    uint64_t fin2 = 0ull;
    bool ok = true;  // warp-uniform
    for (int j = 0; j < ntw; ++j) {
      // ---- S_j out of TMEM; the columns go back to the MMA warp at once ----
      if (!wait_warp(bar(kBarSFull + w), j & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kTileN];
#pragma unroll
      for (int c = 0; c < kTileN / 32; ++c) {
        float v[32];
        tmem_ld32(trow + s_col + 32 * c, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[32 * c + i] = v[i];
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(bar(kBarSFree + w));
      // ---- softmax of this thread's row ---------------------------------------
      const int kp0 = j * kTileN;
      // causal (attention.rs:207): key position <= query position; a masked
      // score is f32::MIN, finite as in the reference, and its ex2 is 0. Only
      // tiles reaching past the tile's first query position need the mask;
      // rows past the tile's tokens read zeros.
      if (kp0 + kTileN - 1 > se.base + qw0 || !live) {
#pragma unroll
        for (int i = 0; i < kTileN; ++i) {
          if (live && kp0 + i > qpos) s[i] = -FLT_MAX;
          if (!live) s[i] = 0.f;
        }
      }
      float mx;
      {  // eight independent chains of three-input maxes (16 scores each)
        float m8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float m = fmax3(s[16 * k], s[16 * k + 1], s[16 * k + 2]);
#pragma unroll
          for (int i = 3; i < 15; i += 2) m = fmax3(m, s[16 * k + i], s[16 * k + i + 1]);
          m8[k] = fmaxf(m, s[16 * k + 15]);
        }
        mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
      }
      // The running max moves only when the row's max grows by more than 2^8.
      const bool grow = mx > m_used + 8.f;
      float corr = 1.f;
      if (grow) {
        corr = ex2(m_used - mx);  // 0 on the first tile
        m_used = mx;
      }
      // x - m and the row sum two lanes at a time (f32x2), four partial sums
      const uint64_t neg_m = pack2(-m_used, -m_used);
      uint64_t ps2[4] = {0ull, 0ull, 0ull, 0ull};  // +0.0f in both lanes
      uint32_t pw[kTileN / 2];  // P row, bf16 pairs
#pragma unroll
      for (int i = 0; i < kTileN / 2; ++i) {
        float xa, xb;
        const uint64_t s2 = pack2(s[2 * i], s[2 * i + 1]);
        unpack2(add2(s2, neg_m), xa, xb);
        fin2 = fma2(s2, 0ull, fin2);  // +0 per finite score, NaN per non-finite one
        const float a = ex2(xa), b = ex2(xb);
        ps2[i & 3] = add2(ps2[i & 3], pack2(a, b));
        pw[i] = bf16x2(a, b);
      }
      float psum;
      {
        float l0, h0;
        unpack2(add2(add2(ps2[0], ps2[1]), add2(ps2[2], ps2[3])), l0, h0);
        psum = l0 + h0;
      }
      l_sum = fmaf(l_sum, corr, psum);
      // ---- P_{j-1} V done: P_w and O_w are free ---------------------------------
      if (j > 0) {
        if (!wait_warp(bar(kBarODone + w), (j - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // tcgen05.ld/st are warp-collective: a warp rescales O when any of its
        // rows moved its max; the other rows scale by 1.
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int c = 0; c < kHeadDim / 32; ++c) {
            float v[32];
            tmem_ld32(trow + o_col + 32 * c, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= corr;
            tmem_st32(trow + o_col + 32 * c, v);
          }
        }
      }
      tmem_st32u(trow + p_col, pw);
      tmem_st32u(trow + p_col + 32, pw + 32);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(bar(kBarPFull + w));
    }
    // ---- epilogue: O / l to the output rows ------------------------------------
    if (ok && ntw > 0) {
      // softmax.rs:17-22,35-40: a non-finite score or row sum fails the
      // sequence's step (its batch rolls it back).
      float f0, f1;
      unpack2(fin2, f0, f1);
      const bool bad = live && !(f0 == 0.f && f1 == 0.f && isfinite(l_sum) && l_sum > 0.f);
      if (__any_sync(0xffffffffu, bad) && lane == 0 && p.status) {
        uint32_t si;  // the grid's y index is the sequence's batch row
        asm volatile("mov.u32 %0, %%ctaid.y;" : "=r"(si));
        atomicOr(&p.status[si], kStatusNonFiniteScore);
      }
      if (!wait_warp(bar(kBarODone + w), (ntw - 1) & 1)) {
        ok = false;
      } else {
        tc_fence_after();
        // every lane loads (warp-collective); live rows store
        const float inv = 1.f / l_sum;
        float* dst = p.out + (static_cast<size_t>(se.row_offset + qw0 + (live ? tq : 0)) * Hq +
                              h * G + gq) * kHeadDim;
#pragma unroll
        for (int c = 0; c < kHeadDim / 32; ++c) {
          float v[32];
          tmem_ld32(trow + o_col + 32 * c, v);
          tmem_wait_ld();
          if (live) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(dst + 32 * c + i) =
                  make_float4(v[i] * inv, v[i + 1] * inv, v[i + 2] * inv, v[i + 3] * inv);
          }
        }
      }
    }
    if (!ok) raise_abort();
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Cfg::kRegsProducer) : "memory");
    const CtaWork cw = cta_work<G, QT>(p);
    const int warp = thread_index() >> 5, lane = thread_index() & 31;  // read again, as cw
    auto raise_abort = [&]() {
      if (lane == 0) {
        st_volatile_shared(sbase + abort_off, 1u);
        atomicOr(p.g.error, kErrTimeout);
      }
    };
    const int h = cw.h, nt0 = cw.nt0, nt1 = cw.nt1, n_kv = cw.n_kv, n_load = cw.n_load;
    const int Hkv = p.g.kv_heads;
    const uint32_t tmem = ld_volatile_shared(sbase + ws_off_misc<QT>());
    const int n_blocks = (n_kv + kBlockTokens - 1) / kBlockTokens;
    // Shared addresses are rederived from sb, made opaque once per tile, so
    // that they are not all held in registers across the loops.
    uint32_t sb = sbase;
    auto pbar = [&](int i) { return sb + Cfg::kOffBar + 8u * static_cast<uint32_t>(i); };
    auto pwait = [&](uint32_t b, uint32_t parity) {
      const bool ok = bar_wait_ab(b, parity, sb + abort_off);
      return __all_sync(0xffffffffu, ok);
    };
    if (warp == kLoadWarp) {
      // ================= loader =================
      // K and V tile t -> stage t % 3: its 16-token blocks through the block
      // table, one lane per block (lanes 0-7); each lane loads the next tile's
      // block id while the current one is copied. A tile is always loaded
      // whole: slots past the sequence's last block take that block again, so
      // every staged V row is a pool row, which is finite (the pool never
      // holds a non-finite value), and a masked P = 0 times it is 0.
      const int32_t* bt = p.g.block_table + static_cast<size_t>(cw.se.slot) * p.g.max_blocks_per_seq;
      const int layer_row0 = p.layer * p.g.num_blocks * Hkv;
      auto block_id = [&](int t) {
        const int b = min(t * (kTileN / kBlockTokens) + lane, n_blocks - 1);
        return (lane < kTileN / kBlockTokens) ? bt[b] : 0;
      };
      int blk_next = block_id(0);
      int k_issued = 0, v_issued = 0;
      bool ok = true;
      for (int t = 0; t < n_load; ++t) {
        sb = opaque(sb);
        const int st = t % kWsStages;
        int32_t blk = blk_next;
        blk_next = block_id(t + 1);
        constexpr int nb = kTileN / kBlockTokens;
        if (static_cast<uint32_t>(blk) >= static_cast<uint32_t>(p.g.num_blocks)) {
          if (lane < nb) atomicOr(p.g.error, kErrBadBlock);
          blk = 0;
        }
        const int y = (layer_row0 + blk * Hkv + h) * kBlockTokens;
        const uint32_t off = static_cast<uint32_t>(st * kTileBytes + lane * kBlockTokens * 128);
        const uint32_t bytes = static_cast<uint32_t>(nb) * kBlockTokens * kHeadDim * 2;
        const uint32_t free_parity = static_cast<uint32_t>((t / kWsStages - 1) & 1);
        if (t >= kWsStages && !pwait(pbar(kBarKFree + st), free_parity)) {
          ok = false;
          break;
        }
        if (lane == 0) bar_expect_tx(pbar(kBarKFull + st), bytes);
        __syncwarp();
        if (lane < nb) tma_rows(sb + Cfg::kOffK + off, &p.tmap_k, y, pbar(kBarKFull + st));
        __syncwarp();
        k_issued = t + 1;
        if (t >= kWsStages && !pwait(pbar(kBarVFree + st), free_parity)) {
          ok = false;
          break;
        }
        if (lane == 0) bar_expect_tx(pbar(kBarVFull + st), bytes);
        __syncwarp();
        if (lane < nb) tma_rows(sb + Cfg::kOffV + off, &p.tmap_v, y, pbar(kBarVFull + st));
        __syncwarp();
        v_issued = t + 1;
      }
      if (!ok) raise_abort();
      // Every copy this warp issued lands before the CTA's shared memory is
      // released, also when another role gave up and left it unread (a copy
      // the MMA warp consumed has completed its phase: no wait).
      for (int t = max(0, k_issued - kWsStages); t < k_issued; ++t)
        bar_wait(pbar(kBarKFull + t % kWsStages), (t / kWsStages) & 1);
      for (int t = max(0, v_issued - kWsStages); t < v_issued; ++t)
        bar_wait(pbar(kBarVFull + t % kWsStages), (t / kWsStages) & 1);
      __syncwarp();
    } else if (warp == kSWarp || warp == kPvWarp) {
      // ============ MMA issue: warp 9 the S products, warp 10 the P V products ============
      // (lane 0 issues; the warp waits together). Two issuers, so that the
      // next S of one query tile never queues behind the other tile's P V.
      constexpr uint32_t kIdQK = idesc(kTileM, kTileN, false);
      constexpr uint32_t kIdPV = idesc(kTileM, kHeadDim, true);
      auto issue_s = [&](int w, int t) {  // S_w = Q_w K_t^T
        if (lane == 0) {
          const uint32_t kaddr = sb + Cfg::kOffK + (t % kWsStages) * kTileBytes;
          const uint32_t qaddr = sb + Cfg::kOffQ + w * kTileBytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16(tmem + w * kTileN, sdesc(qaddr + 32 * kk, 1, 64), sdesc(kaddr + 32 * kk, 1, 64),
                    kIdQK, kk > 0);
          mma_commit(pbar(kBarSFull + w));
        }
      };
      auto issue_pv = [&](int w, int t) {  // O_w += P_w V_t, P_w from TMEM
        if (lane == 0) {
          const uint32_t vaddr = sb + Cfg::kOffV + (t % kWsStages) * kTileBytes;
#pragma unroll
          for (int kk = 0; kk < kTileN / 16; ++kk)  // 16 tokens = 8 P columns a step
            mma_f16_ts(tmem + Cfg::kOCol + w * kHeadDim, tmem + Cfg::kPCol + w * (kTileN / 2) + 8 * kk,
                       sdesc(vaddr + 2048 * kk, kTileBytes >> 4, 64), kIdPV, (t > 0 || kk > 0) ? 1 : 0);
          mma_commit(pbar(kBarODone + w));
        }
      };
      auto commit_to = [&](int b) {
        if (lane == 0) mma_commit(bar(b));
      };
      // V_t landed; on the last tile, rows past the cache are cleared: P is 0
      // there, but 0 times a non-finite stale value is not 0.
      auto v_ready = [&](int t) {
        if (!pwait(pbar(kBarVFull + t % kWsStages), (t / kWsStages) & 1)) return false;
        const int valid = n_kv - t * kTileN;
        if (valid < kTileN) {
          uint8_t* vt = sm + Cfg::kOffV + (t % kWsStages) * kTileBytes;
          // row t of a swizzled tile is the 128 bytes at t*128 (units permuted)
          for (int i = valid * 8 + lane; i < kTileN * 8; i += 32)
            *reinterpret_cast<uint4*>(vt + (i >> 3) * 128 + (i & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
        }
        return true;
      };
      bool ok = true;
      if (warp == kSWarp) {
        ok = pwait(pbar(kBarQFull + 0), 0) && (nt1 == 0 || pwait(pbar(kBarQFull + 1), 0));
        for (int j = 0; ok && j < n_load; ++j) {
          sb = opaque(sb);
          if (!pwait(pbar(kBarKFull + j % kWsStages), (j / kWsStages) & 1)) {
            ok = false;
            break;
          }
          // S_w,j overwrites S_w,j-1: it goes once warpgroup w has read that
          if (j < nt0) {
            if (j > 0 && !pwait(pbar(kBarSFree + 0), (j - 1) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(0, j);
          }
          if (j < nt1) {
            if (j > 0 && !pwait(pbar(kBarSFree + 1), (j - 1) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(1, j);
          }
          commit_to(kBarKFree + j % kWsStages);
        }
      } else {
        for (int j = 0; ok && j < n_load; ++j) {
          sb = opaque(sb);
          bool have_v = false;
          if (j < nt0) {
            if (!pwait(pbar(kBarPFull + 0), j & 1) || !v_ready(j)) {
              ok = false;
              break;
            }
            have_v = true;
            tc_fence_after();
            issue_pv(0, j);
          }
          if (j < nt1) {
            if (!pwait(pbar(kBarPFull + 1), j & 1) || (!have_v && !v_ready(j))) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(1, j);
          }
          commit_to(kBarVFree + j % kWsStages);
        }
      }
      if (!ok) raise_abort();
      // every MMA this warp issued completes before TMEM is released
      commit_to(kBarDrain + (warp - kSWarp));
      bar_wait(pbar(kBarDrain + (warp - kSWarp)), 0);
      __syncwarp();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kSWarp)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                     ld_volatile_shared(sbase + ws_off_misc<QT>())),
                 "r"(Cfg::kTmemCols)
                 : "memory");
}

}  // namespace

bool prefill_tc_supported(const PrefillLaunch& p) {
  const int G = p.g.q_heads / p.g.kv_heads;
  return p.g.bf16 && (G == 1 || G == 2 || G == 4 || G == 8);
}

cudaError_t launch_prefill_tc(const PrefillLaunch& p, cudaStream_t s) {
  if (p.n_seq <= 0 || p.max_count <= 0) return cudaSuccess;
  using Cfg = WsCfg<kPrefillQT>;
  const int G = p.g.q_heads / p.g.kv_heads;
  const int tq = kPrefillQT * (kTileM / G);  // new tokens per CTA
  const int n_tiles = (p.max_count + tq - 1) / tq;
  if (n_tiles > 65535 || p.n_seq > 65535) return cudaErrorInvalidConfiguration;  // grid y/z limits
  const dim3 grid(p.g.kv_heads, p.n_seq, n_tiles);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static unsigned long long configured[4] = {};  // per G variant, one bit per device
  auto run = [&](auto kernel, int gi) {
    if (dev < 64 && !(configured[gi] & (1ull << dev))) {
      // setmaxnreg.inc waits until the CTA's launch registers cover the
      // split; a build that launched with fewer would never get them.
      cudaFuncAttributes fa{};
      cudaError_t a = cudaFuncGetAttributes(&fa, kernel);
      if (a != cudaSuccess) return a;
      if (fa.numRegs < Cfg::kRegsLaunch) return cudaErrorInvalidConfiguration;
      a = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               ws_smem<kPrefillQT>());
      if (a != cudaSuccess) return a;
      configured[gi] |= (1ull << dev);
    }
    kernel<<<grid, Cfg::kThreads, ws_smem<kPrefillQT>(), s>>>(p);
    return cudaGetLastError();
  };
  switch (G) {
    case 1: return run(prefill_ws_kernel<1, kPrefillQT>, 0);
    case 2: return run(prefill_ws_kernel<2, kPrefillQT>, 1);
    case 4: return run(prefill_ws_kernel<4, kPrefillQT>, 2);
    case 8: return run(prefill_ws_kernel<8, kPrefillQT>, 3);
    default: return cudaErrorInvalidValue;
  }
}

SLMKV_TL_SETTER(timeline_set_prefill_tc)

}  // namespace slmkv
