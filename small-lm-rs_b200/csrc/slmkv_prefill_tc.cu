// Causal GQA prefill attention over a bf16 paged cache on the 5th-generation
// tensor cores (tcgen05): the batched prompt path of
// ProjectedQkv::{scaled_causal_scores, causal_probabilities, attend_values}
// (rust/engine/src/attention.rs:195-399) with the cache of
// forward_prefill_with_cache (attention.rs:835-870).
//
// One CTA = 128 query rows of one (sequence, KV head): the G query heads of
// the group times 128/G consecutive new tokens (row r = token r/G, head r%G),
// so every K/V tile is shared by the whole group. Per 128-token K/V tile:
//   S = Q K^T        tcgen05.mma kind::f16, M=128 N=128, f32 in TMEM columns
//                    [0,128); Q rounded to bf16 after RoPE and scaling
//   softmax          4 warps, one row per thread (TMEM lane = row), exp2
//                    domain, causal mask; the running max moves only when a
//                    row's max grows by more than 2^8, then O is rescaled
//   O += P V         M=128 N=64, P (bf16) from shared memory, V as an
//                    MN-major operand, O in TMEM columns [128,192)
// Q, K and V tiles are 128-byte-swizzled: K/V blocks arrive by TMA (16 rows
// per block, block-table lookups; two tiles in flight), Q and P are written
// by the threads in the same layout. One thread issues the MMAs and commits
// them to mbarriers. Two CTAs share an SM (112 KiB of shared memory and 256
// TMEM columns each), so one CTA's softmax overlaps the other's MMAs and
// copies. Every wait is bounded; on expiry the CTA records an error, waits
// (bounded) for its own MMAs and copies, frees TMEM and exits.
#include <cstdint>

#include "slmkv_internal.h"

namespace slmkv {
namespace {

constexpr int kTileM = 128;    // query rows per CTA
constexpr int kTileN = 128;    // K/V tokens per tile (8 blocks)
constexpr int kTmemCols = 256; // S: [0,128), O: [128,192)
constexpr int kOCol = 128;
constexpr int kTileBytes = kTileN * kHeadDim * 2;  // 16 KiB: 128 rows of 128 B
constexpr float kScaleLog2Tc = 0.125f * 1.4426950408889634f;
constexpr unsigned long long kWaitNs = 1000000000ull;  // 1 s
constexpr int kWaitSpinsMax = 1 << 26;

// Shared memory. The dynamic base is the start of the CTA's window (the
// kernel has no static shared variables), 1024-aligned as the 128-byte
// swizzle needs; the kernel checks it and reports an error otherwise.
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTileBytes;            // 2 buffers
constexpr int kOffV = kOffK + 2 * kTileBytes;        // 2 buffers
constexpr int kOffP = kOffV + 2 * kTileBytes;        // tokens 0-63, 64-127
constexpr int kOffBar = kOffP + 2 * kTileBytes;      // k_full[2], v_full[2], s_done, o_done
constexpr int kOffMisc = kOffBar + 6 * 8;            // TMEM base address
constexpr int kSmemTc = kOffMisc + 16;
static_assert(2 * (kSmemTc + 1024) <= 228 * 1024, "two prefill CTAs must fit one SM");

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
__device__ __noinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
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

template <int G>
__global__ void __launch_bounds__(128, 2) prefill_tc_kernel(const __grid_constant__ PrefillLaunch p) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const uint32_t sbase = su32(sm);
  if (sbase & 1023u) {  // uniform over the CTA: report instead of misreading tiles
    if (threadIdx.x == 0) atomicOr(p.g.error, kErrLayout);
    return;
  }
  const int tid = threadIdx.x, warp = tid >> 5;
  const int si = blockIdx.y, h = blockIdx.z;
  const int tile = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);  // long tiles first
  constexpr int TQ = kTileM / G;  // new tokens per CTA
  const SeqEntry se = p.seqs[si];
  const int q0 = tile * TQ;
  if (q0 >= se.count) return;
  const int nq = min(TQ, se.count - q0);
  const int Hkv = p.g.kv_heads, Hq = p.g.q_heads;
  const int last_pos = se.base + q0 + nq - 1;
  const int n_kv = last_pos + 1;
  const int n_tiles = (n_kv + kTileN - 1) / kTileN;

  const uint32_t bar_k0 = sbase + kOffBar, bar_v0 = sbase + kOffBar + 16,
                 bar_s = sbase + kOffBar + 32, bar_o = sbase + kOffBar + 40;
  uint32_t* misc = reinterpret_cast<uint32_t*>(sm + kOffMisc);
  if (tid == 0) {
    bar_init(bar_k0, 1);
    bar_init(bar_k0 + 8, 1);
    bar_init(bar_v0, 1);
    bar_init(bar_v0 + 8, 1);
    bar_init(bar_s, 1);
    bar_init(bar_o, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     sbase + kOffMisc),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }

  // K or V tile j -> buffer j&1: its 16-token blocks through the block table,
  // by warp 0 with one lane per block (the table lookups overlap). K tile j+2
  // goes as soon as S_j has been read out of TMEM, V tile j+1 as soon as
  // P·V_{j-1} is done, so copies run a tile or two ahead.
  const int32_t* bt = p.g.block_table + static_cast<size_t>(se.slot) * p.g.max_blocks_per_seq;
  const int layer_row0 = p.layer * p.g.num_blocks * Hkv;
  const int lane = tid & 31;
  const int n_blocks = (n_kv + kBlockTokens - 1) / kBlockTokens;
  // Block ids of tiles [win, win+8) in warp 0's registers: blk_cur holds
  // tiles win..win+3 (lane l: tile win + l/8, block l%8), blk_nxt the next
  // four. The window moves at the top of an iteration, when the oldest tile
  // still needed (V of tile j+1) has left its first half; the next four
  // tiles' ids then load four iterations before they are needed.
  int win = 0, blk_cur = 0, blk_nxt = 0;
  auto fetch_window = [&](int first_tile) {
    const int b = first_tile * (kTileN / kBlockTokens) + lane;
    return b < n_blocks ? bt[b] : 0;
  };
  if (warp == 0) {
    blk_cur = fetch_window(0);
    blk_nxt = fetch_window(4);
  }
  auto advance_window = [&](int oldest) {  // warp 0
    while (oldest >= win + 4) {
      blk_cur = blk_nxt;
      win += 4;
      blk_nxt = fetch_window(win + 4);
    }
  };
  auto block_of = [&](int t, int b) {  // warp 0, all lanes; win <= t < win + 8
    const int rel = t - win;
    const int a = __shfl_sync(0xffffffffu, blk_cur, ((rel & 3) << 3) + b);
    const int c = __shfl_sync(0xffffffffu, blk_nxt, ((rel & 3) << 3) + b);
    return rel < 4 ? a : c;
  };
  auto load_half = [&](int j, bool v) {  // warp 0, all lanes
    const int b0 = j * (kTileN / kBlockTokens);
    const int nb = min(kTileN / kBlockTokens, n_blocks - b0);
    const uint32_t bar = (v ? bar_v0 : bar_k0) + 8 * (j & 1);
    int32_t blk = block_of(j, lane & 7);
    if (lane == 0) bar_expect_tx(bar, static_cast<uint32_t>(nb) * kBlockTokens * kHeadDim * 2);
    __syncwarp();
    if (lane < nb) {
      if (static_cast<uint32_t>(blk) >= static_cast<uint32_t>(p.g.num_blocks)) {
        atomicOr(p.g.error, kErrBadBlock);
        blk = 0;
      }
      const int y = (layer_row0 + blk * Hkv + h) * kBlockTokens;
      const uint32_t off = static_cast<uint32_t>((j & 1) * kTileBytes + lane * kBlockTokens * 128);
      tma_rows(sbase + (v ? kOffV : kOffK) + off, v ? &p.tmap_v : &p.tmap_k, y, bar);
    }
    __syncwarp();
  };

  // Q rows: RoPE at the token's position, scaled into the exp2 domain, bf16
  // (hi, lo); rows past the CTA's tokens are zero.
  const int r = tid;  // this thread's row (TMEM lane)
  const int tq = r / G, gq = r % G;
  const int qpos = se.base + q0 + tq;
  {
    uint8_t* qt = sm + kOffQ;
    const bool live = tq < nq;
    const float2* src = reinterpret_cast<const float2*>(
        p.q + (static_cast<size_t>(se.row_offset + q0 + (live ? tq : 0)) * Hq + h * G + gq) *
                  kHeadDim);
    const float2* cs = p.g.rope + static_cast<size_t>(live ? qpos : 0) * (kHeadDim / 2);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      uint32_t hw[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float2 x = live ? src[4 * u + k] : make_float2(0.f, 0.f);
        if (live && p.rotate) {
          const float2 c = cs[4 * u + k];
          x = make_float2(__fsub_rn(__fmul_rn(x.x, c.x), __fmul_rn(x.y, c.y)),
                          __fadd_rn(__fmul_rn(x.x, c.y), __fmul_rn(x.y, c.x)));
        }
        x.x *= kScaleLog2Tc;
        x.y *= kScaleLog2Tc;
        hw[k] = bf16x2(x.x, x.y);
      }
      *reinterpret_cast<uint4*>(qt + swz(r, u)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  const uint32_t tmem_row = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  constexpr uint32_t kIdQK = idesc(kTileM, kTileN, false);
  constexpr uint32_t kIdPV = idesc(kTileM, kHeadDim, true);
  // Progress (thread 0's view), for draining on an error: K and V tiles
  // whose copies were issued / seen landed, S and P·V products issued / seen.
  int k_issued = 0, k_seen = 0, v_issued = 0, v_seen = 0, s_issued = 0, s_seen = 0,
      o_issued = 0, o_seen = 0;
  // A failed wait sets this thread's flag; the CTA decides at its barriers
  // with __syncthreads_or, so every thread takes the same branch.
  bool fail = false;
  auto issue_s = [&](int j) {  // thread 0: S_j = Q K_j^T once K_j landed
    if (!bar_wait(bar_k0 + 8 * (j & 1), (j >> 1) & 1)) {
      fail = true;
      return;
    }
    k_seen = j + 1;
    tc_fence_after();
    const uint32_t kaddr = sbase + kOffK + (j & 1) * kTileBytes;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      mma_f16(tmem, sdesc(sbase + kOffQ + 32 * kk, 1, 64), sdesc(kaddr + 32 * kk, 1, 64), kIdQK,
              kk > 0);
    mma_commit(bar_s);
    s_issued = j + 1;
  };
  if (warp == 0) {
    for (int t = 0; t < min(n_tiles, 2); ++t) {
      load_half(t, false);
      load_half(t, true);
    }
    k_issued = v_issued = min(n_tiles, 2);
    if (lane == 0) issue_s(0);
  }

  float m_used = -INFINITY, l_sum = 0.f;
  bool aborted = false;
  for (int j = 0; j < n_tiles; ++j) {
    const int buf = j & 1;
    const uint32_t vaddr = sbase + kOffV + buf * kTileBytes;
    if (warp == 0) advance_window(j + 1);
    // ---- S_j out of TMEM into registers ----------------------------------------
    if (!bar_wait(bar_s, j & 1)) fail = true;
    else if (tid == 0) s_seen = j + 1;
    tc_fence_after();
    float s[kTileN];
#pragma unroll
    for (int c = 0; c < kTileN / 32; ++c) {
      float v[32];
      tmem_ld32(tmem_row + 32 * c, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) s[32 * c + i] = v[i];
    }
    tmem_wait_ld();
    tc_fence_before();
    aborted = __syncthreads_or(fail) != 0;
    tc_fence_after();
    if (aborted) break;
    // S columns and K buffer j&1 are free: the next copy and product start now.
    if (warp == 0) {
      if (j + 2 < n_tiles) {
        load_half(j + 2, false);
        k_issued = j + 3;
      }
      if (lane == 0 && j + 1 < n_tiles) issue_s(j + 1);
    }
    // ---- softmax of this thread's row ---------------------------------------
    const bool live = tq < nq;
    const int kp0 = j * kTileN;
    float mx = -INFINITY;
    // causal (attention.rs:207): key position <= query position. Only tiles
    // reaching past the CTA's first query position need the mask (the same
    // decision in every thread); rows past the CTA's tokens read zeros.
    if (kp0 + kTileN - 1 > se.base + q0 || !live) {
#pragma unroll
      for (int i = 0; i < kTileN; ++i) {
        if (live && kp0 + i > qpos) s[i] = -INFINITY;
        if (!live) s[i] = 0.f;
      }
    }
    {  // eight independent chains instead of one 128-long dependency chain
      float m8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) m8[k] = s[k];
#pragma unroll
      for (int i = 8; i < kTileN; ++i) m8[i & 7] = fmaxf(m8[i & 7], s[i]);
      mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                 fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
    }
    const bool grow = mx > m_used + 8.f;
    float corr = 1.f;
    if (grow) {
      corr = ex2(m_used - mx);  // 0 on the first tile
      m_used = mx;
    }
    float ps8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // independent partial sums
    uint32_t pw[kTileN / 2];
#pragma unroll
    for (int i = 0; i < kTileN / 2; ++i) {
      const float a = ex2(s[2 * i] - m_used), b = ex2(s[2 * i + 1] - m_used);
      ps8[i & 7] += a + b;
      pw[i] = bf16x2(a, b);
    }
    const float psum = ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
    l_sum = fmaf(l_sum, corr, psum);
    // ---- P·V_{j-1} done: P, O and V buffer (j-1)&1 are free ------------------
    if (j > 0) {
      const bool o_ok = bar_wait(bar_o, (j - 1) & 1);
      if (!o_ok) fail = true;
      if (warp == 0 && __all_sync(0xffffffffu, o_ok)) {
        o_seen = j;
        if (j + 1 < n_tiles) {
          load_half(j + 1, true);
          v_issued = j + 2;
        }
      }
    }
    tc_fence_after();
    // tcgen05.ld/st are warp-collective (.sync.aligned): a warp rescales O
    // when any of its rows moved its max; the other rows scale by 1.
    if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
      for (int c = 0; c < kHeadDim / 32; ++c) {
        float v[32];
        tmem_ld32(tmem_row + kOCol + 32 * c, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= corr;
        tmem_st32(tmem_row + kOCol + 32 * c, v);
      }
      tmem_wait_st();
    }
    uint8_t* prow = sm + kOffP;
#pragma unroll
    for (int u = 0; u < kTileN / 8; ++u)  // tokens 0-63 in the first P tile, 64-127 in the second
      *reinterpret_cast<uint4*>(prow + (u >> 3) * kTileBytes + swz(r, u & 7)) =
          make_uint4(pw[4 * u], pw[4 * u + 1], pw[4 * u + 2], pw[4 * u + 3]);
    const int valid = min(kTileN, n_kv - kp0);
    if (valid < kTileN) {
      // The last tile: P = 0 past the cache, but 0 times a non-finite stale
      // value is not 0. Clear those V rows once the tile landed.
      if (!bar_wait(bar_v0 + 8 * buf, (j >> 1) & 1)) fail = true;
      uint8_t* vt = sm + kOffV + buf * kTileBytes;
      // row t of a swizzled tile is the 128 bytes at t*128 (units permuted)
      for (int i = valid * 8 + tid; i < kTileN * 8; i += 128)
        *reinterpret_cast<uint4*>(vt + (i >> 3) * 128 + (i & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    aborted = __syncthreads_or(fail) != 0;
    tc_fence_after();
    if (aborted) break;
    // ---- O += P V ----------------------------------------------------------------
    if (tid == 0) {
      if (bar_wait(bar_v0 + 8 * buf, (j >> 1) & 1)) {
        v_seen = j + 1;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTileN / 16; ++kk)
          mma_f16(tmem + kOCol,
                  sdesc(sbase + kOffP + (kk >> 2) * kTileBytes + 32 * (kk & 3), 1, 64),
                  sdesc(vaddr + 2048 * kk, kTileBytes >> 4, 64), kIdPV, (j > 0 || kk > 0) ? 1 : 0);
        mma_commit(bar_o);
        o_issued = j + 1;
      } else {
        fail = true;
      }
    }
  }

  // ---- epilogue: O / l to the output rows --------------------------------------
  tc_fence_before();
  aborted = __syncthreads_or(fail) != 0;
  tc_fence_after();
  if (!aborted) {
    if (!bar_wait(bar_o, (n_tiles - 1) & 1)) fail = true;
    else if (tid == 0) o_seen = n_tiles;
  }
  tc_fence_before();
  const bool abort = __syncthreads_or(fail) != 0;  // the same in every thread
  tc_fence_after();
  if (!abort) {
    // every thread of the warp loads (warp-collective); live rows store
    const float inv = 1.f / l_sum;
    float* dst = p.out + (static_cast<size_t>(se.row_offset + q0 + (tq < nq ? tq : 0)) * Hq + h * G +
                          gq) * kHeadDim;
#pragma unroll
    for (int c = 0; c < kHeadDim / 32; ++c) {
      float v[32];
      tmem_ld32(tmem_row + kOCol + 32 * c, v);
      tmem_wait_ld();
      if (tq < nq) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(dst + 32 * c + i) =
              make_float4(v[i] * inv, v[i + 1] * inv, v[i + 2] * inv, v[i + 3] * inv);
      }
    }
  } else if (tid == 0) {
    atomicOr(p.g.error, kErrTimeout);
    // Let this CTA's own MMAs and copies land (bounded) before its TMEM and
    // shared memory are released.
    if (s_issued > s_seen) bar_wait(bar_s, (s_issued - 1) & 1);
    if (o_issued > o_seen) bar_wait(bar_o, (o_issued - 1) & 1);
    for (int t = k_seen; t < k_issued; ++t) bar_wait(bar_k0 + 8 * (t & 1), (t >> 1) & 1);
    for (int t = v_seen; t < v_issued; ++t) bar_wait(bar_v0 + 8 * (t & 1), (t >> 1) & 1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                 : "memory");
}

}  // namespace

bool prefill_tc_supported(const PrefillLaunch& p) {
  const int G = p.g.q_heads / p.g.kv_heads;
  return p.g.bf16 && (G == 1 || G == 2 || G == 4 || G == 8);
}

cudaError_t launch_prefill_tc(const PrefillLaunch& p, cudaStream_t s) {
  if (p.n_seq <= 0 || p.max_count <= 0) return cudaSuccess;
  const int G = p.g.q_heads / p.g.kv_heads;
  const int tq = kTileM / G;
  const dim3 grid((p.max_count + tq - 1) / tq, p.n_seq, p.g.kv_heads);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static unsigned long long configured[4] = {};  // per G variant, one bit per device
  auto run = [&](auto kernel, int gi) {
    if (dev < 64 && !(configured[gi] & (1ull << dev))) {
      const cudaError_t a =
          cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc);
      if (a != cudaSuccess) return a;
      configured[gi] |= (1ull << dev);
    }
    kernel<<<grid, 128, kSmemTc, s>>>(p);
    return cudaGetLastError();
  };
  switch (G) {
    case 1: return run(prefill_tc_kernel<1>, 0);
    case 2: return run(prefill_tc_kernel<2>, 1);
    case 4: return run(prefill_tc_kernel<4>, 2);
    case 8: return run(prefill_tc_kernel<8>, 3);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace slmkv
