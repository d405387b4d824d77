// sm_100a kernels of the KV-cache hot path.
//
//   append_kernel    KvCache::append_layer (kv_cache.rs:182-230) with the K
//                    half of RoPE (rope.rs:82-100) fused into the store.
//   decode_kernel    GroupedQueryAttention::forward_cached_token's cache part
//                    (attention.rs:794-810): RoPE(Q, K) at the pre-append
//                    position, the paged append, and attend_cached_query
//                    (attention.rs:677-759) as split-K online softmax.
//   prefill_kernel   causal attention of a step's new tokens over the cache
//                    (attention.rs:195-399 when the cache starts empty).
//   gather_kernel    KvCache::layer_keys/layer_values (kv_cache.rs:237-248).
//   apply_updates    block-table writes and copy-on-write block copies.
//
// Paged pool layout: [layer][block][kv_head][slot 0..15][d=64], f32 or bf16.
// One (layer, block, kv_head) chunk is 4 KiB (f32) / 2 KiB (bf16) and
// contiguous, so a decode CTA stages it with one cp.async.bulk per chunk.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "slmkv_internal.h"
#include "slmkv_libm.h"

namespace slmkv {
namespace {

constexpr int D = kHeadDim;
constexpr unsigned kFull = 0xffffffffu;
// 1/sqrt(64) * log2(e): scores are kept in the exp2 domain.
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // bounded waits: 1 s

// ---------------------------------------------------------------------------
// PTX helpers: mbarrier + bulk async copy (the TMA engine, non-tensor form).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Global -> shared bulk copy completing on `bar`; 16-byte aligned addresses,
// size a multiple of 16 (every chunk here is 2 or 4 KiB at chunk offsets).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// TMA tiled load of a 2-D box at column 0, row y (no multicast).
__device__ __forceinline__ void tma_load_rows(void* dst, const CUtensorMap* map, int y,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits for phase `parity` of `bar` for at most ~1 s (and a fixed iteration
// cap); returns false when the limit ran out.
__device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  for (uint32_t i = 0; i < (1u << 24); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31u) == 0 && globaltimer_ns() - start > kWaitLimitNs) break;
  }
  return false;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity);
}

// Counter arrival with release and acquire at gpu scope, and the relaxed
// store that resets a counter for the next launch.
__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void st_relaxed(int* p, int v) {
  asm volatile("st.relaxed.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 2^x on the MUFU unit (scores live in the exp2 domain); ex2(-inf) = +0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------------------
// Numerics shared with the reference.
// ---------------------------------------------------------------------------
// rope.rs:94-97 — separately rounded products, no FMA contraction.
__device__ __forceinline__ float2 rope_pair(float2 x, float2 cs) {
  const float a = __fmul_rn(x.x, cs.x), b = __fmul_rn(x.y, cs.y);
  const float e = __fmul_rn(x.x, cs.y), f = __fmul_rn(x.y, cs.x);
  return make_float2(__fsub_rn(a, b), __fadd_rn(e, f));
}
// linear.rs:14-23 round-to-nearest-even, returning the 16 kept bits.
__device__ __forceinline__ uint32_t bf16_bits(float x) {
  const uint32_t b = __float_as_uint(x);
  if (!isfinite(x)) return (b >> 16) | ((x != x) ? 0x0040u : 0u);  // keep NaN a NaN
  return (b + 0x7fffu + ((b >> 16) & 1u)) >> 16;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return bf16_bits(lo) | (bf16_bits(hi) << 16);
}
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ bool finite2(float2 v) { return isfinite(v.x) && isfinite(v.y); }
// softmax.rs:17-22: a score row with a non-finite entry is rejected. True when
// one of this lane's G scores is not finite and its token is a real one.
template <int G>
__device__ __forceinline__ bool scores_bad(const float (&sc)[G], bool valid) {
  bool bad = false;
#pragma unroll
  for (int g = 0; g < G; ++g) bad |= !isfinite(sc[g]);
  return valid && bad;
}
__device__ __forceinline__ bool finite4(float4 v) {
  return isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
}
// Both halves of a bf16 pair finite (a finite f32 near FLT_MAX rounds to inf).
__device__ __forceinline__ bool finite_bf16x2(uint32_t w) {
  return (w & 0x7f80u) != 0x7f80u && (w & 0x7f800000u) != 0x7f800000u;
}

// Q rows live in shared memory as 16 four-float units per head; unit u is
// stored at u ^ ((u >> 3) & 1) so that the rotated unit reads of both the
// f32 and the bf16 score loops are free of bank conflicts.
__device__ __forceinline__ int qunit(int u) { return u ^ ((u >> 3) & 1); }

__device__ __forceinline__ int32_t checked_block(const PoolGeom& g, int32_t blk) {
  if (static_cast<uint32_t>(blk) >= static_cast<uint32_t>(g.num_blocks)) {
    atomicOr(g.error, kErrBadBlock);
    return 0;
  }
  return blk;
}

// ---------------------------------------------------------------------------
// Score of one 16-token block against G query heads, per lane.
// Lane l handles token t = l & 15 and dims [32*(l>>4), +32); the two halves
// are combined with one shuffle. K is read in a rotated chunk order so that
// the 8 lanes of each quarter-warp hit 8 distinct bank groups.
// ---------------------------------------------------------------------------
template <int G>
__device__ __forceinline__ void block_scores_f32(const float* __restrict__ kb,
                                                 const float* __restrict__ qs, int lane,
                                                 float (&sc)[G]) {
  const int t = lane & 15, hh = lane >> 4;
  const float* krow = kb + t * D + hh * 32;
  float a0[G], a1[G];  // two chains per head halve the dependent FMA depth
#pragma unroll
  for (int g = 0; g < G; ++g) a0[g] = a1[g] = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int c = (j + t) & 7;
    const float4 k4 = *reinterpret_cast<const float4*>(krow + 4 * c);
    const int pu = qunit(hh * 8 + c);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float4 q4 = *reinterpret_cast<const float4*>(qs + g * D + pu * 4);
      a0[g] = fmaf(q4.x, k4.x, a0[g]);
      a1[g] = fmaf(q4.y, k4.y, a1[g]);
      a0[g] = fmaf(q4.z, k4.z, a0[g]);
      a1[g] = fmaf(q4.w, k4.w, a1[g]);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    sc[g] = a0[g] + a1[g];
    sc[g] += __shfl_xor_sync(kFull, sc[g], 16);
  }
}

template <int G>
__device__ __forceinline__ void block_scores_bf16(const uint16_t* __restrict__ kb,
                                                  const float* __restrict__ qs, int lane,
                                                  float (&sc)[G]) {
  const int t = lane & 15, hh = lane >> 4;
  const uint16_t* krow = kb + t * D;
  float a0[G], a1[G];
#pragma unroll
  for (int g = 0; g < G; ++g) a0[g] = a1[g] = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = (2 * j + hh + t) & 7;  // chunk of 8 dims
    const uint4 raw = *reinterpret_cast<const uint4*>(krow + 8 * c);
    const float k0 = bf16lo(raw.x), k1 = bf16hi(raw.x), k2 = bf16lo(raw.y), k3 = bf16hi(raw.y);
    const float k4 = bf16lo(raw.z), k5 = bf16hi(raw.z), k6 = bf16lo(raw.w), k7 = bf16hi(raw.w);
    const int p0 = qunit(2 * c), p1 = qunit(2 * c + 1);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float4 qa = *reinterpret_cast<const float4*>(qs + g * D + p0 * 4);
      const float4 qb = *reinterpret_cast<const float4*>(qs + g * D + p1 * 4);
      a0[g] = fmaf(qa.x, k0, a0[g]);
      a1[g] = fmaf(qa.y, k1, a1[g]);
      a0[g] = fmaf(qa.z, k2, a0[g]);
      a1[g] = fmaf(qa.w, k3, a1[g]);
      a0[g] = fmaf(qb.x, k4, a0[g]);
      a1[g] = fmaf(qb.y, k5, a1[g]);
      a0[g] = fmaf(qb.z, k6, a0[g]);
      a1[g] = fmaf(qb.w, k7, a1[g]);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    sc[g] = a0[g] + a1[g];
    sc[g] += __shfl_xor_sync(kFull, sc[g], 16);
  }
}

// Online-softmax update for one block, then P·V (lane owns dims 2l, 2l+1).
// sc: raw dot products for token lane&15; nvalid >= 1 tokens are real.
// pbuf: this warp's G*16 floats of shared memory for the probabilities.
// Rows at or past nvalid are never multiplied (they may hold stale data).
template <int G, bool BF16V>
__device__ __forceinline__ void block_softmax_pv(const void* __restrict__ vb, float* pbuf, int lane,
                                                 int nvalid, const float (&sc)[G], float (&m)[G],
                                                 float (&l)[G], float2 (&acc)[G]) {
  const int t = lane & 15;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float s = (t < nvalid) ? sc[g] * kScaleLog2 : -INFINITY;
    float mb = s;
    mb = fmaxf(mb, __shfl_xor_sync(kFull, mb, 8));
    mb = fmaxf(mb, __shfl_xor_sync(kFull, mb, 4));
    mb = fmaxf(mb, __shfl_xor_sync(kFull, mb, 2));
    mb = fmaxf(mb, __shfl_xor_sync(kFull, mb, 1));
    const float mnew = fmaxf(m[g], mb);  // finite: nvalid >= 1
    const float corr = fast_exp2(m[g] - mnew);
    const float p = fast_exp2(s - mnew);
    if (lane < 16) pbuf[g * 16 + t] = p;
    float ps = p;
    ps += __shfl_xor_sync(kFull, ps, 8);
    ps += __shfl_xor_sync(kFull, ps, 4);
    ps += __shfl_xor_sync(kFull, ps, 2);
    ps += __shfl_xor_sync(kFull, ps, 1);
    l[g] = fmaf(l[g], corr, ps);
    acc[g].x *= corr;
    acc[g].y *= corr;
    m[g] = mnew;
  }
  __syncwarp();
  auto vrow = [&](int tt) {
    if constexpr (BF16V) {
      const uint32_t w = reinterpret_cast<const uint32_t*>(vb)[tt * (D / 2) + lane];
      return make_float2(bf16lo(w), bf16hi(w));
    } else {
      return reinterpret_cast<const float2*>(vb)[tt * (D / 2) + lane];
    }
  };
  if (nvalid == kBlockTokens) {
#pragma unroll
    for (int t4 = 0; t4 < kBlockTokens; t4 += 4) {
      const float2 v0 = vrow(t4), v1 = vrow(t4 + 1), v2 = vrow(t4 + 2), v3 = vrow(t4 + 3);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4 p4 = *reinterpret_cast<const float4*>(pbuf + g * 16 + t4);
        acc[g].x = fmaf(p4.x, v0.x, acc[g].x);
        acc[g].y = fmaf(p4.x, v0.y, acc[g].y);
        acc[g].x = fmaf(p4.y, v1.x, acc[g].x);
        acc[g].y = fmaf(p4.y, v1.y, acc[g].y);
        acc[g].x = fmaf(p4.z, v2.x, acc[g].x);
        acc[g].y = fmaf(p4.z, v2.y, acc[g].y);
        acc[g].x = fmaf(p4.w, v3.x, acc[g].x);
        acc[g].y = fmaf(p4.w, v3.y, acc[g].y);
      }
    }
  } else {
    for (int tt = 0; tt < nvalid; ++tt) {
      const float2 v2 = vrow(tt);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pt = pbuf[g * 16 + tt];
        acc[g].x = fmaf(pt, v2.x, acc[g].x);
        acc[g].y = fmaf(pt, v2.y, acc[g].y);
      }
    }
  }
  __syncwarp();  // pbuf is rewritten by the next block
}

// Maximum of v over the warp in one instruction (sm_100a).
__device__ __forceinline__ float warp_max(float v) {
  float r;
  asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off);
  return v;
}

// block_softmax_pv for f32 V as the decode kernel runs it: the block's
// maximum in one warp reduction, and the row sum l kept per lane (lane t < 16
// holds its tokens' share, lanes 16-31 hold 0) so that no block waits on a
// sum reduction; warp_sum(l) at the end of the segment gives the total.
template <int G>
__device__ __forceinline__ void block_softmax_pv_lanesum(const float* __restrict__ vb, float* pbuf,
                                                         int lane, int nvalid, const float (&sc)[G],
                                                         float (&m)[G], float (&l)[G],
                                                         float2 (&acc)[G]) {
  const int t = lane & 15;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float s = (t < nvalid) ? sc[g] * kScaleLog2 : -INFINITY;
    const float mnew = fmaxf(m[g], warp_max(s));  // finite: nvalid >= 1
    const float corr = fast_exp2(m[g] - mnew);
    const float p = fast_exp2(s - mnew);
    if (lane < 16) pbuf[g * 16 + t] = p;
    l[g] = fmaf(l[g], corr, (lane < 16) ? p : 0.f);
    acc[g].x *= corr;
    acc[g].y *= corr;
    m[g] = mnew;
  }
  __syncwarp();
  const float2* v2 = reinterpret_cast<const float2*>(vb);
  if (nvalid == kBlockTokens) {
#pragma unroll
    for (int t4 = 0; t4 < kBlockTokens; t4 += 4) {
      const float2 v0 = v2[t4 * (D / 2) + lane], v1 = v2[(t4 + 1) * (D / 2) + lane];
      const float2 w2 = v2[(t4 + 2) * (D / 2) + lane], w3 = v2[(t4 + 3) * (D / 2) + lane];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4 p4 = *reinterpret_cast<const float4*>(pbuf + g * 16 + t4);
        acc[g].x = fmaf(p4.x, v0.x, acc[g].x);
        acc[g].y = fmaf(p4.x, v0.y, acc[g].y);
        acc[g].x = fmaf(p4.y, v1.x, acc[g].x);
        acc[g].y = fmaf(p4.y, v1.y, acc[g].y);
        acc[g].x = fmaf(p4.z, w2.x, acc[g].x);
        acc[g].y = fmaf(p4.z, w2.y, acc[g].y);
        acc[g].x = fmaf(p4.w, w3.x, acc[g].x);
        acc[g].y = fmaf(p4.w, w3.y, acc[g].y);
      }
    }
  } else {
    for (int tt = 0; tt < nvalid; ++tt) {
      const float2 vv = v2[tt * (D / 2) + lane];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pt = pbuf[g * 16 + tt];
        acc[g].x = fmaf(pt, vv.x, acc[g].x);
        acc[g].y = fmaf(pt, vv.y, acc[g].y);
      }
    }
  }
  __syncwarp();  // pbuf is rewritten by the next block
}

// ---------------------------------------------------------------------------
// bf16 K/V blocks on the tensor cores (warp-level mma.m16n8k16, f32
// accumulate). The block's K and V chunks are staged by TMA with the 128-byte
// swizzle: row r (a token, 64 bf16 = 128 B) lies at (r/8)*1024 + (r%8)*128,
// its 16-byte unit u at unit u ^ (r%8), so ldmatrix reads are conflict-free.
// The 16 MMA rows hold the G query heads twice: row g is head g rounded to
// bf16, row g+8 the bf16 residual of the same values, so Q (and P) carry ~16
// mantissa bits and every sum is accumulated in f32. Lane (g = lane/4,
// t = lane%4) owns head g (when g < G): scores of tokens 8j+2t+{0,1}, j=0,1,
// and outputs of dims 8n+2t+{0,1}, n=0..7 (hi row in o[n][0..1], residual row
// in o[n][2..3]).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t sw128(uint32_t base, int row, int unit) {
  return base + ((row >> 3) << 10) + ((row & 7) << 7) + (((unit ^ row) & 7) << 4);
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// (hi, lo) bf16 pairs of two f32 values: hi = RNE(x), lo = RNE(x - hi).
__device__ __forceinline__ void split_bf16x2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16x2(x0, x1);
  lo = pack_bf16x2(__fsub_rn(x0, bf16lo(hi)), __fsub_rn(x1, bf16hi(hi)));
}

// Q fragments of one pair: qs holds the pair's rotated Q rows [G][64] (f32);
// each is scaled into the exp2 domain and split into (hi, lo) bf16.
template <int G>
__device__ __forceinline__ void load_q_frags(const float* qs, int lane, uint32_t (&qa)[4][4]) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    if (g < G) {
      const float2 x = *reinterpret_cast<const float2*>(qs + g * D + 16 * s + 2 * t);
      const float2 y = *reinterpret_cast<const float2*>(qs + g * D + 16 * s + 8 + 2 * t);
      split_bf16x2(x.x * kScaleLog2, x.y * kScaleLog2, qa[s][0], qa[s][1]);
      split_bf16x2(y.x * kScaleLog2, y.y * kScaleLog2, qa[s][2], qa[s][3]);
    } else {
      qa[s][0] = qa[s][1] = qa[s][2] = qa[s][3] = 0u;
    }
  }
}

// One block: scores on the tensor cores, the online-softmax update for this
// lane's head, then P·V on the tensor cores. kaddr/vaddr: shared addresses of
// the swizzled K and V chunks; tokens at or past nvalid are masked (their V
// rows must be finite: the caller zeroes them). l_row accumulates this lane's
// share of the row sum: the caller adds the quad's shares at the segment end.
__device__ __forceinline__ void block_mma_bf16(uint32_t kaddr, uint32_t vaddr, int lane, int nvalid,
                                               const uint32_t (&qa)[4][4], float& m_row,
                                               float& l_row, float (&o)[8][4], bool& bad) {
  const int r = lane & 7, mtx = lane >> 3, t = lane & 3;
  float c[2][4];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.f;
#pragma unroll
    for (int sp = 0; sp < 2; ++sp) {
      uint32_t b0, b1, b2, b3;  // k-steps 2sp (b0, b1) and 2sp+1 (b2, b3)
      ldsm_x4(sw128(kaddr, 8 * j + r, 4 * sp + mtx), b0, b1, b2, b3);
      mma_bf16(c[j], qa[2 * sp][0], qa[2 * sp][1], qa[2 * sp][2], qa[2 * sp][3], b0, b1);
      mma_bf16(c[j], qa[2 * sp + 1][0], qa[2 * sp + 1][1], qa[2 * sp + 1][2], qa[2 * sp + 1][3],
               b2, b3);
    }
  }
  float sc[2][2];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int tok = 8 * j + 2 * t + e;
      const float v = c[j][e] + c[j][2 + e];
      bad |= (tok < nvalid) && !isfinite(v);  // softmax.rs:17-22
      sc[j][e] = (tok < nvalid) ? v : -INFINITY;
      mx = fmaxf(mx, sc[j][e]);
    }
  mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
  const float mnew = fmaxf(m_row, mx);
  const float corr = fast_exp2(m_row - mnew);
  float pr[2][2], ps = 0.f;
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      pr[j][e] = fast_exp2(sc[j][e] - mnew);
      ps += pr[j][e];
    }
  l_row = fmaf(l_row, corr, ps);  // this lane's share; the quad's sum at the segment's end
  m_row = mnew;
  uint32_t pa0, pa1, pa2, pa3;
  split_bf16x2(pr[0][0], pr[0][1], pa0, pa1);
  split_bf16x2(pr[1][0], pr[1][1], pa2, pa3);
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    o[n][0] *= corr;
    o[n][1] *= corr;
    o[n][2] *= corr;
    o[n][3] *= corr;
  }
#pragma unroll
  for (int np = 0; np < 4; ++np) {
    uint32_t b0, b1, b2, b3;  // dims 16np..+7 (b0, b1) and 16np+8..+15 (b2, b3)
    ldsm_x4_t(sw128(vaddr, 8 * (mtx & 1) + r, 2 * np + (mtx >> 1)), b0, b1, b2, b3);
    mma_bf16(o[2 * np], pa0, pa1, pa2, pa3, b0, b1);
    mma_bf16(o[2 * np + 1], pa0, pa1, pa2, pa3, b2, b3);
  }
}

// ---------------------------------------------------------------------------
// Decode (stream-K). The host flattens the step into a stream of chunk ids
// (chunk = physical block * Hkv + kv head; one chunk = 16 tokens of one head)
// in (sequence, head, block) order, plus one PairEntry per (sequence, head).
// Every warp of the persistent grid takes an equal slice [g0, g1) of that
// stream and works alone: lane 0 keeps R bulk copies (K chunk + V chunk per
// stage) in flight ahead of the warp's own consumption, refilling each stage
// as soon as the warp has consumed it; no barrier is shared between warps.
// A (sequence, head) whose blocks span several warps is merged by the last
// warp to finish it (atomic counter, no waiting).
// ---------------------------------------------------------------------------
template <int BF16, int G, int W, int R>
struct StreamShape {
  static constexpr int kEsz = BF16 ? 2 : 4;
  static constexpr int kChunk = kBlockTokens * D * kEsz;  // one block of one head, K or V
  static constexpr int kStage = 2 * kChunk;
  // Side buffer of a stage: the pair's Q rows, its RoPE row and its new K/V
  // rows, copied together with the pair's first block in this warp.
  static constexpr int kSideCs = G * D * 4;
  static constexpr int kSideKn = kSideCs + (D / 2) * 8;
  static constexpr int kSideVn = kSideKn + D * 4;
  static constexpr int kSide = kSideVn + D * 4;
  static constexpr int kSlot = ((G * D * 4 + G * 8) + 15) / 16 * 16;  // one segment partial
  static constexpr int kOffSide = W * R * kStage;
  static constexpr int kOffQ = kOffSide + W * R * kSide;
  static constexpr int kOffP = kOffQ + W * G * D * 4;
  static constexpr int kOffSlots = kOffP + W * G * kBlockTokens * 4;
  static constexpr int kOffBars = kOffSlots + 2 * W * kSlot;
  static constexpr int kOffChunk = kOffBars + W * R * 8;
  static constexpr int kOffCnt = kOffChunk + W * R * 4;  // 3 x 2W merge-slot counters
  static constexpr int kOffPend = (kOffCnt + 6 * W * 4 + 15) / 16 * 16;
  // Per warp: its start record (2 x int4) and the cross-CTA pairs it has
  // pending in the current layer (2 x int4), kept out of registers.
  static constexpr int kOffRec = kOffPend + W * R * 16;
  static constexpr int kSmem = kOffRec + W * 64 + (BF16 ? 1024 : 0);  // + alignment slack
  static_assert(kSmem <= 227 * 1024, "decode staging exceeds shared memory");
  static_assert(kChunk % 16 == 0 && kSide % 16 == 0 && kSlot % 16 == 0, "16-byte alignment");
};

struct PairFields {
  int seq, head, L, blk_begin, nblk, part_base, first_warp, nseg;
  int at_warp_start;  // the pair's first block is its first warp's first block
};

__device__ __forceinline__ PairFields pair_from_window(const int4& a, const int4& b, int k) {
  PairFields f;
  f.seq = __shfl_sync(kFull, a.x, k);
  f.head = __shfl_sync(kFull, a.y, k);
  f.L = __shfl_sync(kFull, a.z, k);
  f.blk_begin = __shfl_sync(kFull, a.w, k);
  f.nblk = __shfl_sync(kFull, b.x, k);
  f.part_base = __shfl_sync(kFull, b.y, k);
  f.first_warp = __shfl_sync(kFull, b.z, k);
  const int ns = __shfl_sync(kFull, b.w, k);
  f.nseg = ns & 0x3fffffff;
  f.at_warp_start = (ns >> 30) & 1;
  return f;
}

// Merges n segment partials (each G x (acc[64], (m, l))) for this lane's two
// output dims: partial s is weighted by 2^(m_s - M), summed in slot order.
// acc_at(s, g) / ml_at(s, g) read one partial. The (m, l) pairs of up to 32
// partials are loaded lane-parallel and the first four partials' acc rows are
// loaded before any of them is used, so a merge of up to four partials (the
// common case) waits for one round of loads, whatever G.
template <int G, typename Acc, typename Ml>
__device__ __forceinline__ void merge_partials(int n, int lane, Acc acc_at, Ml ml_at, float2 (&A)[G],
                                               float (&Mo)[G], float (&Lo)[G]) {
  float M[G], Ls[G];
  float2 a2[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    M[g] = -INFINITY;
    Ls[g] = 0.f;
    a2[g] = make_float2(0.f, 0.f);
  }
  for (int base = 0; base < n; base += 32) {
    const int cnt = min(32, n - base);
    float2 mine[G];
#pragma unroll
    for (int g = 0; g < G; ++g)
      mine[g] = (lane < cnt) ? ml_at(base + lane, g) : make_float2(-INFINITY, 0.f);
    float2 a[4][G];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int g = 0; g < G; ++g) a[u][g] = (u < cnt) ? acc_at(base + u, g) : make_float2(0.f, 0.f);
    float fmine[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float Mc = mine[g].x;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) Mc = fmaxf(Mc, __shfl_xor_sync(kFull, Mc, off));
      const float Mn = fmaxf(M[g], Mc);
      const float rescale = exp2f(M[g] - Mn);  // M = -inf on the first chunk: 0
      a2[g].x *= rescale;
      a2[g].y *= rescale;
      Ls[g] *= rescale;
      M[g] = Mn;
      fmine[g] = exp2f(mine[g].x - Mn);  // lanes past cnt: 0
      float lsum = mine[g].y * fmine[g];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) lsum += __shfl_xor_sync(kFull, lsum, off);
      Ls[g] += lsum;
    }
    for (int s0 = 0; s0 < cnt; s0 += 4) {
      if (s0 > 0) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int g = 0; g < G; ++g)
            a[u][g] = (s0 + u < cnt) ? acc_at(base + s0 + u, g) : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float f = __shfl_sync(kFull, fmine[g], min(s0 + u, 31));
          if (s0 + u < cnt) {
            a2[g].x = fmaf(a[u][g].x, f, a2[g].x);
            a2[g].y = fmaf(a[u][g].y, f, a2[g].y);
          }
        }
      }
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    A[g] = a2[g];
    Mo[g] = M[g];
    Lo[g] = Ls[g];
  }
}

template <int BF16, int G, int W, int R, bool ML>
__global__ void __launch_bounds__(W * 32, 1)
    decode_stream_kernel(const __grid_constant__ StreamDecodeLaunch p) {
  SLMKV_TL(ML ? kTlDecodeLayers : kTlDecode);
  using Sh = StreamShape<BF16, G, W, R>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // bf16 stages are TMA boxes with the 128-byte swizzle: 1024-byte aligned.
  uint8_t* smem = smem_raw + (BF16 ? ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u) : 0u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* stages = smem + warp * R * Sh::kStage;
  uint8_t* sides = smem + Sh::kOffSide + warp * R * Sh::kSide;
  float* qs = reinterpret_cast<float*>(smem + Sh::kOffQ) + warp * G * D;
  float* pbuf = reinterpret_cast<float*>(smem + Sh::kOffP) + warp * G * kBlockTokens;
  uint8_t* slots = smem + Sh::kOffSlots;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Sh::kOffBars) + warp * R;
  int* stage_chunk = reinterpret_cast<int*>(smem + Sh::kOffChunk) + warp * R;
  // In-CTA merge bookkeeping, per slot: arrivals (at the pair's first slot),
  // partials written into the slot, and partials read out of it by a merge.
  int* cta_cnt = reinterpret_cast<int*>(smem + Sh::kOffCnt);
  int* slot_wr = cta_cnt + 2 * W;
  int* slot_rd = cta_cnt + 4 * W;
  int4* side_pend = reinterpret_cast<int4*>(smem + Sh::kOffPend) + warp * R;
  int4* rec = reinterpret_cast<int4*>(smem + Sh::kOffRec) + warp * 4;

  if (threadIdx.x < 6 * W) cta_cnt[threadIdx.x] = 0;
  const int gw = blockIdx.x * W + warp;
  const bool active = gw < p.n_warps;

  // Start record: {first pair, seq, head, ctx_len}, {first pair's end in the
  // stream, g0, g1, -}; the warp owns stream blocks [g0, g1) (never empty) of
  // every layer of the launch. The step plan (start records, chunk stream,
  // pair entries) is written only by host-to-device copies ordered before the
  // previous kernel of the stream, never by a kernel, so it is read before
  // the wait below.
  int4 r0 = make_int4(0, 0, 0, 0), r1 = r0;
  if (active) {
    r0 = p.warp_start[2 * gw];
    r1 = p.warp_start[2 * gw + 1];
  }
  const int g0 = r1.y, g1 = r1.z;
  if (lane == 0) {  // read back at the layer boundaries
    rec[0] = r0;
    rec[1] = r1;
  }
  // The warp's blocks over the launch: its slice of layer 0, then the same
  // slice of layer 1, and so on (the plan is the same for every layer).
  const int total = ML ? p.n_layers * (g1 - g0) : g1 - g0;
  int cwin = g0;
  int cval = (g0 + lane < g1) ? p.chunks[g0 + lane] : 0;

  // ---- pair window: one PairEntry per lane, shared by producer and consumer --
  int pwin = r0.x;
  int4 pa = make_int4(0, 0, 0, 0), pb = make_int4(0, 0, 0, 0);
  auto load_window = [&](int from) {
    pwin = from;
    if (from + lane < p.n_pairs) {
      const int4* e = reinterpret_cast<const int4*>(p.pairs + from + lane);
      pa = e[0];
      pb = e[1];
    }
  };
  if (active) load_window(r0.x);
  if (active && lane == 0) {
    for (int s = 0; s < R; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  const int cta_w0 = blockIdx.x * W;
  const int cta_w1 = min(cta_w0 + W, p.n_warps) - 1;

  const int Hkv = p.g.kv_heads, Hq = p.g.q_heads;
  const size_t layer_bytes = static_cast<size_t>(p.g.layer_elems) * Sh::kEsz;
  const uint8_t* kbase = static_cast<const uint8_t*>(p.g.k) + p.layer * layer_bytes;
  const uint8_t* vbase = static_cast<const uint8_t*>(p.g.v) + p.layer * layer_bytes;
  const uint32_t max_chunk = static_cast<uint32_t>(p.g.num_blocks) * Hkv;

  // ---- producer: lane 0 keeps R stages in flight ahead of the consumer ------
  int pg = g0, pl = 0, pv = 0;  // next stream block to issue, its layer, blocks issued
  int pp = r0.x, pp_seq = r0.y, pp_head = r0.z, pp_L = r0.w, pp_end = r1.x;
  int pp_first = g0;  // first block of pair pp in this warp
  int pc = r0.x;      // the consumer's pair; the window never moves past it
  // Side copies of a stage that starts a pair (lane 0): the pair's Q rows,
  // its RoPE row and, when this warp ends the pair, the new K/V rows.
  auto issue_side = [&](int stage, int seq, int head, int L, bool appends, int layer) {
    uint8_t* sd = sides + stage * Sh::kSide;
    bulk_load(sd, p.q[ML ? layer : 0] + (static_cast<size_t>(seq) * Hq + head * G) * D, G * D * 4,
              &bars[stage]);
    if (p.fused)
      bulk_load(sd + Sh::kSideCs, p.g.rope + static_cast<size_t>(L - 1) * (D / 2), (D / 2) * 8,
                &bars[stage]);
    if (appends) {
      const size_t row = (static_cast<size_t>(seq) * Hkv + head) * D;
      bulk_load(sd + Sh::kSideKn, p.k_new[ML ? layer : 0] + row, D * 4, &bars[stage]);
      bulk_load(sd + Sh::kSideVn, p.v_new[ML ? layer : 0] + row, D * 4, &bars[stage]);
    }
  };
  // Arms the next stage and copies its K/V chunks; with defer_side the side
  // copies are recorded in side_pend and issued later on the same barrier
  // (its expected byte count already includes them).
  auto issue = [&](int stage, bool defer_side) {
    if (ML && pg == g1) {  // the producer enters the next layer: the slice again
      ++pl;
      pg = g0;
      const int4 a = rec[0];
      pp = a.x;
      pp_seq = a.y;
      pp_head = a.z;
      pp_L = a.w;
      pp_end = rec[1].x;
      pp_first = g0;
      if (cwin != g0) {  // the chunk window is the producer's alone
        cwin = g0;
        cval = (g0 + lane < g1) ? p.chunks[g0 + lane] : 0;
      }
    } else if (pg == pp_end) {  // the producer enters the next pair
      ++pp;
      if (pp - pwin >= 32) load_window(pc);
      const PairFields f = pair_from_window(pa, pb, pp - pwin);
      pp_seq = f.seq;
      pp_head = f.head;
      pp_L = f.L;
      pp_first = f.blk_begin;
      pp_end = f.blk_begin + f.nblk;
    }
    if (pg - cwin >= 32) {
      cwin = pg;
      cval = (pg + lane < g1) ? p.chunks[pg + lane] : 0;
    }
    uint32_t chunk = static_cast<uint32_t>(__shfl_sync(kFull, cval, pg - cwin));
    if (lane == 0) {
      if (chunk >= max_chunk) {
        atomicOr(p.g.error, kErrBadBlock);
        chunk = 0;
      }
      stage_chunk[stage] = static_cast<int>(chunk);
      uint8_t* st = stages + stage * Sh::kStage;
      const bool first = (pg == pp_first);
      const bool appends = p.fused && first && (pp_end - 1 < g1);
      uint32_t tx = Sh::kStage;
      if (first) tx += G * D * 4 + (p.fused ? (D / 2) * 8 : 0) + (appends ? 2 * D * 4 : 0);
      mbar_arrive_expect_tx(&bars[stage], tx);
      if constexpr (BF16) {
        const int y = ((p.layer + pl) * static_cast<int>(max_chunk) + static_cast<int>(chunk)) *
                      kBlockTokens;
        tma_load_rows(st, &p.tmap_k, y, &bars[stage]);
        tma_load_rows(st + Sh::kChunk, &p.tmap_v, y, &bars[stage]);
      } else {
        const size_t off = pl * layer_bytes + static_cast<size_t>(chunk) * Sh::kChunk;
        bulk_load(st, kbase + off, Sh::kChunk, &bars[stage]);
        bulk_load(st + Sh::kChunk, vbase + off, Sh::kChunk, &bars[stage]);
      }
      if (defer_side)
        side_pend[stage] = first ? make_int4(pp_seq, pp_head, pp_L, (pl << 1) | (appends ? 1 : 0))
                                 : make_int4(0, 0, 0, -1);
      else if (first)
        issue_side(stage, pp_seq, pp_head, pp_L, appends, pl);
    }
    ++pg;
    ++pv;
  };

  // The first stages' K/V may be fetched before waiting on the previous
  // kernel when the host says this layer's pool region was complete before
  // that kernel started (the previous kernel is a decode of another layer).
  if (active && p.early_kv)
    for (int s = 0; s < R && pv < total; ++s) issue(s, true);

  // Launched with programmatic stream serialization: everything above ran
  // while the previous kernel of the stream was finishing; wait for it (and
  // its memory) before touching the step's inputs, the outputs or the split-K
  // scratch. Then everything before this kernel in the stream is complete and
  // visible, and the next kernel may launch: its CTAs start on the SMs this
  // kernel's CTAs leave, and run their own prologue meanwhile.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __syncthreads();  // the only CTA-wide barrier; the warps are independent after it
  if (!active) return;
  SLMKV_TL_MARK(kTlDecodeWaited);
  if (p.early_kv) {
    if (lane == 0)
      for (int s = 0; s < pv; ++s) {
        const int4 e = side_pend[s];
        if (e.w >= 0) issue_side(s, e.x, e.y, e.z, (e.w & 1) != 0, e.w >> 1);
      }
  } else {
    for (int s = 0; s < R && pv < total; ++s) issue(s, false);
  }
  // An output row (one query head of one sequence): f32, and for a one-layer
  // launch that asks for it also as bf16 (linear.rs:14-23 rounding), the next
  // projection's operand.
  auto store_out = [&](float* out, size_t row, float2 v) {
    reinterpret_cast<float2*>(out + row * D)[lane] = v;
    if (!ML && p.out_bf16) p.out_bf16[row * (D / 2) + lane] = pack_bf16x2(v.x, v.y);
  };
  // ---- consumer --------------------------------------------------------------
  PairFields cur = pair_from_window(pa, pb, pc - pwin);
  float m[G], l[G];
  float2 acc[G];
  // bf16: this lane's head (lane/4) on the tensor cores until the segment ends.
  uint32_t qa[4][4];
  float m_row = -INFINITY, l_row = 0.f, o[8][4];
  float2 cs = make_float2(1.f, 0.f), kn = cs, vn = cs;
  int seg_end = min(g1, cur.blk_begin + cur.nblk);
  bool seg_start = true;
  // A score of this segment that is not finite (a non-finite or overflowing
  // query, softmax.rs:17-22): the pair's sequence is flagged at the segment's
  // end and its step fails as attention.rs:731,814-815 does.
  bool bad = false;
  int cl = 0;  // the consumer's layer (of the launch)

  // Cross-CTA pairs of the current layer, merged after its last block (at most two).
  // rec[2 + k]: {pair, global slot base, n CTA segs, row} of pending pair k.
  int npend = 0;

  for (int v = 0, g = g0; v < total; ++v) {
    const int stage = v % R;
    const uint32_t parity = static_cast<uint32_t>(v / R) & 1u;
    if (!mbar_wait_bounded(&bars[stage], parity)) {
      // A copy did not land within the limit: record it, give the copies
      // still in flight a bounded chance to land, and stop this warp.
      if (lane == 0) {
        atomicOr(p.g.error, kErrTimeout);
        for (int c = v + 1; c < pv; ++c)
          mbar_wait_bounded(&bars[c % R], static_cast<uint32_t>(c / R) & 1u);
      }
      __syncwarp();
      return;
    }
    uint8_t* kb = stages + stage * Sh::kStage;
    uint8_t* vb = kb + Sh::kChunk;
    if (seg_start) {
      // Pair inputs arrived with this stage: rotate Q at the new token's
      // position into the swizzled Q buffer; keep the RoPE pair and new K/V.
      const uint8_t* sd = sides + stage * Sh::kSide;
      if (p.fused) {
        cs = reinterpret_cast<const float2*>(sd + Sh::kSideCs)[lane];
        if (cur.blk_begin + cur.nblk - 1 < g1) {
          kn = reinterpret_cast<const float2*>(sd + Sh::kSideKn)[lane];
          vn = reinterpret_cast<const float2*>(sd + Sh::kSideVn)[lane];
        }
      }
#pragma unroll
      for (int g2 = 0; g2 < G; ++g2) {
        float2 x = reinterpret_cast<const float2*>(sd)[g2 * (D / 2) + lane];
        if (p.fused) x = rope_pair(x, cs);
        if constexpr (BF16)
          reinterpret_cast<float2*>(qs + g2 * D)[lane] = x;
        else
          *reinterpret_cast<float2*>(qs + g2 * D + qunit(lane >> 1) * 4 + ((2 * lane) & 3)) = x;
        m[g2] = -INFINITY;
        l[g2] = 0.f;
        acc[g2] = make_float2(0.f, 0.f);
      }
      __syncwarp();
      if constexpr (BF16) {
        load_q_frags<G>(qs, lane, qa);
        m_row = -INFINITY;
        l_row = 0.f;
#pragma unroll
        for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      }
      seg_start = false;
    }
    const int j = g - cur.blk_begin;
    const int tok0 = j * kBlockTokens;
    const int nvalid = min(kBlockTokens, cur.L - tok0);
    const bool append_here = p.fused && (j == cur.nblk - 1);
    if (append_here) {
      // The append: rotate the new key at position L-1, store K/V (rounded
      // to the pool's type) into the staged block and into the pool.
      const int slot = (cur.L - 1) - tok0;
      bool fin = finite2(kn) && finite2(vn);
      float2 kx = rope_pair(kn, cs);
      const size_t dst = static_cast<size_t>(p.layer + cl) * p.g.layer_elems +
                         (static_cast<size_t>(stage_chunk[stage]) * kBlockTokens + slot) * D;
      // Non-finite K/V are stored as zeros: the pool never holds a non-finite
      // value (the step fails and the slot stays past the length).
      if constexpr (BF16) {
        uint32_t kq = pack_bf16x2(kx.x, kx.y), vq = pack_bf16x2(vn.x, vn.y);
        fin = fin && finite_bf16x2(kq) && finite_bf16x2(vq);
        if (!fin) kq = vq = 0u;
        // lane's word: unit lane/4 of the swizzled row `slot`
        const uint32_t off = sw128(0u, slot, lane >> 2) + ((lane & 3) << 2);
        *reinterpret_cast<uint32_t*>(kb + off) = kq;
        *reinterpret_cast<uint32_t*>(vb + off) = vq;
        reinterpret_cast<uint32_t*>(static_cast<uint16_t*>(p.g.k) + dst)[lane] = kq;
        reinterpret_cast<uint32_t*>(static_cast<uint16_t*>(p.g.v) + dst)[lane] = vq;
      } else {
        const float2 vx = fin ? vn : make_float2(0.f, 0.f);
        if (!fin) kx = make_float2(0.f, 0.f);
        reinterpret_cast<float2*>(kb)[slot * (D / 2) + lane] = kx;
        reinterpret_cast<float2*>(vb)[slot * (D / 2) + lane] = vx;
        reinterpret_cast<float2*>(static_cast<float*>(p.g.k) + dst)[lane] = kx;
        reinterpret_cast<float2*>(static_cast<float*>(p.g.v) + dst)[lane] = vx;
      }
      if (!__all_sync(kFull, fin) && lane == 0) atomicOr(&p.status[cur.seq], kStatusNonFinite);
      __syncwarp();
    }
    if constexpr (BF16) {
      if (nvalid < kBlockTokens) {
        // Tokens past the length are masked, but P = 0 times a non-finite
        // stale V value is not 0: clear those V rows (whole 128-byte rows).
        for (int i = nvalid * 8 + lane; i < kBlockTokens * 8; i += 32)
          reinterpret_cast<uint4*>(vb)[((i >> 3) >> 3) * 64 + ((i >> 3) & 7) * 8 + (i & 7)] =
              make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
      }
      block_mma_bf16(smem_u32(kb), smem_u32(vb), lane, nvalid, qa, m_row, l_row, o, bad);
      __syncwarp();
    } else {
      float sc[G];
      block_scores_f32<G>(reinterpret_cast<const float*>(kb), qs, lane, sc);
      bad |= scores_bad<G>(sc, (lane & 15) < nvalid);
      block_softmax_pv_lanesum<G>(reinterpret_cast<const float*>(vb), pbuf, lane, nvalid, sc, m,
                                  l, acc);
    }
    if (pv < total) {
      // The stage (and its side buffer) were read, maybe written, through
      // the generic proxy; order that before the async-proxy refill.
      if (append_here || (BF16 && nvalid < kBlockTokens))
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(stage, false);
    }

    if (g == seg_end - 1) {
      // ---- end of this warp's segment of pair `pc` -------------------------------
      if (__any_sync(kFull, bad)) {
        if (lane == 0 && p.status) atomicOr(&p.status[cur.seq], kStatusNonFiniteScore);
        bad = false;
      }
      if constexpr (!BF16) {
#pragma unroll
        for (int g2 = 0; g2 < G; ++g2) l[g2] = warp_sum(l[g2]);  // the lanes' shares
      }
      if constexpr (BF16) {
        // Back to one float2 per lane and head (dims 2*lane, 2*lane+1): the
        // layout the merges below use. qs is free: Q lives in qa.
        const int gl = lane >> 2, tl = lane & 3;
        if (gl < G) {
#pragma unroll
          for (int n = 0; n < 8; ++n)
            *reinterpret_cast<float2*>(qs + gl * D + 8 * n + 2 * tl) =
                make_float2(o[n][0] + o[n][2], o[n][1] + o[n][3]);
        }
        __syncwarp();
        l_row += __shfl_xor_sync(kFull, l_row, 1);  // the quad's shares of its row sum
        l_row += __shfl_xor_sync(kFull, l_row, 2);
#pragma unroll
        for (int g2 = 0; g2 < G; ++g2) {
          acc[g2] = reinterpret_cast<const float2*>(qs + g2 * D)[lane];
          m[g2] = __shfl_sync(kFull, m_row, 4 * g2);
          l[g2] = __shfl_sync(kFull, l_row, 4 * g2);
        }
        __syncwarp();
      }
      float* out = p.out[ML ? cl : 0];
      const size_t orow = static_cast<size_t>(cur.seq) * Hq + cur.head * G;
      if (cur.nseg == 1) {
#pragma unroll
        for (int g2 = 0; g2 < G; ++g2) {
          const float inv = 1.0f / l[g2];
          store_out(out, orow + g2, make_float2(acc[g2].x * inv, acc[g2].y * inv));
        }
      } else {
        // Warps [ka, kb] of this CTA hold the pair's segments here; they merge
        // in shared memory, the last one to arrive does the merge.
        const int last_warp = cur.first_warp + cur.nseg - 1;
        const int ka = max(cur.first_warp, cta_w0), kbw = min(last_warp, cta_w1);
        const bool whole_in_cta = (cur.first_warp >= cta_w0) && (last_warp <= cta_w1);
        const int n_in = kbw - ka + 1;
        // A segment sits in slot 2k+0 when it is warp k's first segment: true
        // for every warp after ka (the pair started before them); for ka it
        // depends on where the pair starts.
        const int ka_off = (cur.first_warp < cta_w0 || cur.at_warp_start) ? 0 : 1;
        auto seg_slot = [&](int w) { return 2 * (w - cta_w0) + ((w == ka) ? ka_off : 0); };
        float2 A[G];
        float Mo[G], Lo[G];
        bool merged = false;
        if (n_in == 1) {
#pragma unroll
          for (int g2 = 0; g2 < G; ++g2) {
            A[g2] = acc[g2];
            Mo[g2] = m[g2];
            Lo[g2] = l[g2];
          }
          merged = true;
        } else {
          const int my = seg_slot(gw);
          uint8_t* mine = slots + my * Sh::kSlot;
          // A slot is written again (the same pair in a later layer of the
          // launch) only after the merge that read its last partial is done.
          if (ML && lane == 0) {
            const int written = slot_wr[my];
            const uint64_t t0 = globaltimer_ns();
            for (uint32_t i = 0; *reinterpret_cast<volatile int*>(&slot_rd[my]) != written; ++i)
              if ((i & 31u) == 31u && globaltimer_ns() - t0 > kWaitLimitNs) {
                atomicOr(p.g.error, kErrTimeout);
                break;
              }
            __threadfence_block();
          }
          __syncwarp();
#pragma unroll
          for (int g2 = 0; g2 < G; ++g2) {
            reinterpret_cast<float2*>(mine)[g2 * (D / 2) + lane] = acc[g2];
            if (lane == 0)
              reinterpret_cast<float2*>(mine + G * D * 4)[g2] = make_float2(m[g2], l[g2]);
          }
          __threadfence_block();
          __syncwarp();
          int last = 0;
          if (lane == 0) {
            if (ML) slot_wr[my] += 1;
            last = (atomicAdd(&cta_cnt[seg_slot(ka)], 1) == n_in - 1);
          }
          last = __shfl_sync(kFull, last, 0);
          if (last) {
            __threadfence_block();
            auto acc_at = [&](int s, int g2) {
              const uint8_t* sl = slots + seg_slot(ka + s) * Sh::kSlot;
              return reinterpret_cast<const float2*>(sl)[g2 * (D / 2) + lane];
            };
            auto ml_at = [&](int s, int g2) {
              const uint8_t* sl = slots + seg_slot(ka + s) * Sh::kSlot;
              return reinterpret_cast<const float2*>(sl + G * D * 4)[g2];
            };
            merge_partials<G>(n_in, lane, acc_at, ml_at, A, Mo, Lo);
            // Every read of the slots is done: reset the arrivals, release them.
            __threadfence_block();
            __syncwarp();
            if (ML && lane == 0) {
              cta_cnt[seg_slot(ka)] = 0;
              __threadfence_block();
              for (int s = 0; s < n_in; ++s) atomicAdd(&slot_rd[seg_slot(ka + s)], 1);
            }
            merged = true;
          }
        }
        if (merged) {
          if (whole_in_cta) {
#pragma unroll
            for (int g2 = 0; g2 < G; ++g2) {
              const float inv = 1.0f / Lo[g2];
              store_out(out, orow + g2, make_float2(A[g2].x * inv, A[g2].y * inv));
            }
          } else {
            // This CTA's share of a pair that spans CTAs: one global partial
            // (each layer of the launch has its own slots and counters).
            const int first_cta = cur.first_warp / W;
            const int n_cta = last_warp / W - first_cta + 1;
            const size_t gslot = static_cast<size_t>(cl) * p.part_stride + cur.part_base +
                                 (blockIdx.x - first_cta);
#pragma unroll
            for (int g2 = 0; g2 < G; ++g2) {
              reinterpret_cast<float2*>(p.part_acc + (gslot * G + g2) * D)[lane] = A[g2];
              if (lane == 0) p.part_ml[gslot * G + g2] = make_float2(Mo[g2], Lo[g2]);
            }
            const int4 e = make_int4(pc, cur.part_base, n_cta, static_cast<int>(orow));
            if (lane == 0) rec[2 + npend] = e;
            ++npend;
          }
        }
      }
      if (g + 1 < g1) {
        ++pc;
        if (pc - pwin >= 32) load_window(pc);
        cur = pair_from_window(pa, pb, pc - pwin);
        seg_end = min(g1, cur.blk_begin + cur.nblk);
        seg_start = true;
      }
    }
    if (g + 1 < g1) {
      ++g;
      continue;
    }

    // ---- end of this layer's slice: pairs that span CTAs ----------------------
    SLMKV_TL_MARK(kTlDecodeSliceDone);
    // The last CTA to arrive merges the partials. Release this warp's
    // partials, then arrive on each pair's counter (both arrivals in flight
    // together); the next layer's first copies are already in flight.
    if (npend > 0) {
      int* counters = p.counters + static_cast<size_t>(cl) * p.counter_stride;
      // The warp barrier orders every lane's partial writes before lane 0's
      // arrival, whose release (gpu scope, cumulative) publishes them; the
      // arrival's acquire, passed on by the shuffle, orders the last CTA's
      // reads of the other partials after every earlier arrival.
      __syncwarp();
      const int4 pend0 = rec[2], pend1 = rec[3];
      int lastmask = 0;
      if (lane == 0) {
        const int prev0 = atom_add_acq_rel(&counters[pend0.x], 1);
        const int prev1 = (npend > 1) ? atom_add_acq_rel(&counters[pend1.x], 1) : 0;
        if (prev0 == pend0.z - 1) {
          lastmask |= 1;
          st_relaxed(&counters[pend0.x], 0);  // ready for the next launch
        }
        if (npend > 1 && prev1 == pend1.z - 1) {
          lastmask |= 2;
          st_relaxed(&counters[pend1.x], 0);
        }
      }
      lastmask = __shfl_sync(kFull, lastmask, 0);
      if (lastmask != 0) {
        float* out = p.out[ML ? cl : 0];
        const size_t pbase = static_cast<size_t>(cl) * p.part_stride;
        for (int k = 0; k < npend; ++k) {
          if (!((lastmask >> k) & 1)) continue;
          const int4 e = (k == 0) ? pend0 : pend1;
          auto acc_at = [&](int s, int g2) {
            return __ldcg(reinterpret_cast<const float2*>(
                              p.part_acc + ((pbase + e.y + s) * G + g2) * D) + lane);
          };
          auto ml_at = [&](int s, int g2) {
            return __ldcg(&p.part_ml[(pbase + e.y + s) * G + g2]);
          };
          float2 A[G];
          float Mo[G], Lo[G];
          merge_partials<G>(e.z, lane, acc_at, ml_at, A, Mo, Lo);
#pragma unroll
          for (int g2 = 0; g2 < G; ++g2) {
            const float inv = 1.0f / Lo[g2];
            store_out(out, static_cast<size_t>(e.w) + g2, make_float2(A[g2].x * inv, A[g2].y * inv));
          }
        }
      }
      npend = 0;
    }
    if (ML && v + 1 < total) {  // the consumer enters the next layer: the slice again
      ++cl;
      g = g0;
      pc = rec[0].x;
      if (pc < pwin || pc - pwin >= 32) load_window(pc);
      cur = pair_from_window(pa, pb, pc - pwin);
      seg_end = min(g1, cur.blk_begin + cur.nblk);
      seg_start = true;
    }
  }
}

template <int BF16, int G>
cudaError_t launch_decode_t(const StreamDecodeLaunch& p, cudaStream_t s) {
  constexpr int W = decode_warps(BF16, G);
  constexpr int R = decode_stages(BF16, G);
  using Sh = StreamShape<BF16, G, W, R>;
  if (p.total_blocks <= 0) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static unsigned long long configured = 0;  // one bit per device
  if (dev < 64 && !(configured & (1ull << dev))) {
    e = cudaFuncSetAttribute(decode_stream_kernel<BF16, G, W, R, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, Sh::kSmem);
    if constexpr (!BF16)
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(decode_stream_kernel<BF16, G, W, R, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, Sh::kSmem);
    if (e != cudaSuccess) return e;
    configured |= (1ull << dev);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((p.n_warps + W - 1) / W);
  cfg.blockDim = dim3(W * 32);
  cfg.dynamicSmemBytes = Sh::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if constexpr (!BF16) {
    if (p.n_layers > 1)
      return cudaLaunchKernelEx(&cfg, decode_stream_kernel<BF16, G, W, R, true>, p);
  } else {
    if (p.n_layers > 1) return cudaErrorInvalidValue;  // f32 pools only
  }
  return cudaLaunchKernelEx(&cfg, decode_stream_kernel<BF16, G, W, R, false>, p);
}

// ---------------------------------------------------------------------------
// Append: 16 lanes per (token, kv head) row, 4 dims (two RoPE pairs) a lane,
// 128-bit loads and stores.
// ---------------------------------------------------------------------------

// The sequence holding batch token `tok` (the same in every lane): 32 probes a
// round, each round narrowing the range 32-fold (two rounds up to 1024
// sequences).
__device__ __forceinline__ int warp_find_seq(const SeqEntry* seqs, int n, int tok, int lane) {
  int lo = 0, len = n;
  while (len > 1) {
    const int step = (len + 31) >> 5;
    const int idx = lo + lane * step;
    const bool ok = lane * step < len && seqs[idx].row_offset <= tok;
    const unsigned m = __ballot_sync(0xffffffffu, ok);  // lane 0 always holds (offsets ascend from 0)
    const int hit = 31 - __clz(m);
    lo += hit * step;
    len = min(step, len - hit * step);
  }
  return lo;
}

// One CTA appends kAppendRows consecutive (token, KV head) rows: 16 lanes per
// row, four rows per lane group, every K/V load issued before any dependent
// work. Each warp finds the sequence of its first token with a lane-parallel
// search and walks forward from it (its rows span at most a few sequences);
// no CTA barrier.
constexpr int kAppendRowsPerGroup = 4;
constexpr int kAppendRows = 16 * kAppendRowsPerGroup;  // 256 threads = 16 groups of 16

template <int BF16>
__global__ void __launch_bounds__(256) append_kernel(const AppendLaunch p) {
  SLMKV_TL(kTlAppend);
  const int Hkv = p.g.kv_heads;
  const int64_t n_rows = static_cast<int64_t>(p.total_tokens) * Hkv;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kAppendRows;
  const int grp = threadIdx.x >> 4, l16 = threadIdx.x & 15, lane = threadIdx.x & 31;
  float4 kin[kAppendRowsPerGroup], vin[kAppendRowsPerGroup];
#pragma unroll
  for (int j = 0; j < kAppendRowsPerGroup; ++j) {
    const int64_t row = row0 + j * 16 + grp;
    if (row < n_rows) {
      kin[j] = reinterpret_cast<const float4*>(p.k_in + row * D)[l16];
      vin[j] = reinterpret_cast<const float4*>(p.v_in + row * D)[l16];
    }
  }
  // this warp's first row (groups 2w, 2w+1 of 16 rows each)
  const int64_t wrow0 = min(row0 + (grp & ~1), n_rows - 1);
  int si = warp_find_seq(p.seqs, p.n_seq, static_cast<int>(wrow0 / Hkv), lane);
#pragma unroll
  for (int j = 0; j < kAppendRowsPerGroup; ++j) {
    const int64_t row = row0 + j * 16 + grp;
    if (row >= n_rows) break;
    const int tok = static_cast<int>(row / Hkv), h = static_cast<int>(row - static_cast<int64_t>(tok) * Hkv);
    while (si + 1 < p.n_seq && p.seqs[si + 1].row_offset <= tok) ++si;  // rows ascend
    const SeqEntry se = p.seqs[si];
    const int pos = se.base + (tok - se.row_offset);
    const int32_t blk = checked_block(
        p.g, p.g.block_table[static_cast<size_t>(se.slot) * p.g.max_blocks_per_seq +
                             pos / kBlockTokens]);
    float4 k = kin[j];
    const float4 v = vin[j];
    const bool fin = finite4(k) && finite4(v);
    if (p.rotate) {
      const float4 cs =
          reinterpret_cast<const float4*>(p.g.rope + static_cast<size_t>(pos) * (D / 2))[l16];
      const float2 a = rope_pair(make_float2(k.x, k.y), make_float2(cs.x, cs.y));
      const float2 b = rope_pair(make_float2(k.z, k.w), make_float2(cs.z, cs.w));
      k = make_float4(a.x, a.y, b.x, b.y);
    }
    const size_t dst = static_cast<size_t>(p.layer) * p.g.layer_elems +
                       ((static_cast<size_t>(blk) * Hkv + h) * kBlockTokens + pos % kBlockTokens) * D;
    // The pool never holds a non-finite value: a failed append stores zeros
    // (the step is rolled back, the slot stays past the length), so that stale
    // slots a later tile stages are finite and P = 0 times them is 0.
    if constexpr (BF16) {
      uint2 kq = make_uint2(pack_bf16x2(k.x, k.y), pack_bf16x2(k.z, k.w));
      uint2 vq = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
      const bool fq = fin && finite_bf16x2(kq.x) && finite_bf16x2(kq.y) &&
                      finite_bf16x2(vq.x) && finite_bf16x2(vq.y);
      if (!fq) kq = vq = make_uint2(0u, 0u);
      reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.g.k) + dst)[l16] = kq;
      reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.g.v) + dst)[l16] = vq;
      if (!fq) atomicOr(&p.status[si], kStatusNonFinite);
    } else {
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      reinterpret_cast<float4*>(static_cast<float*>(p.g.k) + dst)[l16] = fin ? k : z;
      reinterpret_cast<float4*>(static_cast<float*>(p.g.v) + dst)[l16] = fin ? v : z;
      if (!fin) atomicOr(&p.status[si], kStatusNonFinite);
    }
  }
}

// ---------------------------------------------------------------------------
// Gather: the inverse walk, into dense [length, Hkv, d] f32 (bf16 widens
// exactly).
// ---------------------------------------------------------------------------
template <int BF16>
__global__ void __launch_bounds__(256) gather_kernel(const GatherLaunch p) {
  SLMKV_TL(kTlGather);
  const int Hkv = p.g.kv_heads;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 4;
  const int l16 = threadIdx.x & 15;
  if (row >= p.length * Hkv) return;
  const int pos = row / Hkv, h = row - pos * Hkv;
  const int32_t blk =
      checked_block(p.g, p.g.block_table[static_cast<size_t>(p.slot) * p.g.max_blocks_per_seq +
                                         pos / kBlockTokens]);
  const size_t src = static_cast<size_t>(p.layer) * p.g.layer_elems +
                     ((static_cast<size_t>(blk) * Hkv + h) * kBlockTokens + pos % kBlockTokens) * D;
  float4 k, v;
  if constexpr (BF16) {
    const uint2 kr = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p.g.k) + src)[l16];
    const uint2 vr = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p.g.v) + src)[l16];
    k = make_float4(bf16lo(kr.x), bf16hi(kr.x), bf16lo(kr.y), bf16hi(kr.y));
    v = make_float4(bf16lo(vr.x), bf16hi(vr.x), bf16lo(vr.y), bf16hi(vr.y));
  } else {
    k = reinterpret_cast<const float4*>(static_cast<const float*>(p.g.k) + src)[l16];
    v = reinterpret_cast<const float4*>(static_cast<const float*>(p.g.v) + src)[l16];
  }
  if (p.k_out) reinterpret_cast<float4*>(p.k_out + static_cast<size_t>(row) * D)[l16] = k;
  if (p.v_out) reinterpret_cast<float4*>(p.v_out + static_cast<size_t>(row) * D)[l16] = v;
}

// ---------------------------------------------------------------------------
// Prefill / extend attention on CUDA cores: CTA = (16-query tile, sequence,
// kv head); K/V blocks of the causal range are staged (widened to f32) in
// shared memory; warp w owns query rows w, w+4, w+8, w+12 of the tile.
// ---------------------------------------------------------------------------
template <int BF16, int G>
__global__ void __launch_bounds__(128) prefill_kernel(const PrefillLaunch p) {
  SLMKV_TL(kTlPrefill);
  __shared__ __align__(16) float qs[kBlockTokens * G * D];
  __shared__ __align__(16) float kbuf[kBlockTokens * D];
  __shared__ __align__(16) float vbuf[kBlockTokens * D];
  __shared__ __align__(16) float pbufs[4][G * kBlockTokens];
  const int tile = blockIdx.x, si = blockIdx.y, h = blockIdx.z;
  const SeqEntry se = p.seqs[si];
  const int q0 = tile * kBlockTokens;
  if (q0 >= se.count) return;
  const int nq = min(kBlockTokens, se.count - q0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int Hkv = p.g.kv_heads, Hq = p.g.q_heads;

  for (int i = tid; i < nq * G * (D / 2); i += blockDim.x) {
    const int jq = i / (G * (D / 2));
    const int r = i - jq * G * (D / 2);
    const int g = r / (D / 2), pr = r - g * (D / 2);
    const int row = se.row_offset + q0 + jq;
    const int pos = se.base + q0 + jq;
    float2 x = reinterpret_cast<const float2*>(p.q + (static_cast<size_t>(row) * Hq + h * G + g) * D)[pr];
    if (p.rotate) x = rope_pair(x, p.g.rope[static_cast<size_t>(pos) * (D / 2) + pr]);
    const int u = (2 * pr) >> 2;
    *reinterpret_cast<float2*>(qs + (jq * G + g) * D + qunit(u) * 4 + ((2 * pr) & 3)) = x;
  }

  float m[4][G], l[4][G];
  float2 acc[4][G];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m[r][g] = -INFINITY;
      l[r][g] = 0.f;
      acc[r][g] = make_float2(0.f, 0.f);
    }

  bool bad = false;  // a real score of this tile is not finite (softmax.rs:17-22)
  const int last_pos = se.base + q0 + nq - 1;
  const int nblk = last_pos / kBlockTokens + 1;
  const size_t layer_off = static_cast<size_t>(p.layer) * p.g.layer_elems;
  const int32_t* bt = p.g.block_table + static_cast<size_t>(se.slot) * p.g.max_blocks_per_seq;
  for (int b = 0; b < nblk; ++b) {
    __syncthreads();
    const int32_t blk = checked_block(p.g, bt[b]);
    const size_t off = layer_off + (static_cast<size_t>(blk) * Hkv + h) * (kBlockTokens * D);
    for (int i = tid; i < kBlockTokens * D / 4; i += blockDim.x) {
      float4 k, v;
      if constexpr (BF16) {
        const uint2 kr = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p.g.k) + off)[i];
        const uint2 vr = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p.g.v) + off)[i];
        k = make_float4(bf16lo(kr.x), bf16hi(kr.x), bf16lo(kr.y), bf16hi(kr.y));
        v = make_float4(bf16lo(vr.x), bf16hi(vr.x), bf16lo(vr.y), bf16hi(vr.y));
      } else {
        k = reinterpret_cast<const float4*>(static_cast<const float*>(p.g.k) + off)[i];
        v = reinterpret_cast<const float4*>(static_cast<const float*>(p.g.v) + off)[i];
      }
      reinterpret_cast<float4*>(kbuf)[i] = k;
      reinterpret_cast<float4*>(vbuf)[i] = v;
    }
    __syncthreads();
    const int tok0 = b * kBlockTokens;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int jq = warp + 4 * r;
      if (jq >= nq) break;
      const int qpos = se.base + q0 + jq;
      const int nvalid = min(kBlockTokens, qpos + 1 - tok0);
      if (nvalid <= 0) continue;
      float sc[G];
      block_scores_f32<G>(kbuf, qs + jq * G * D, lane, sc);
      bad |= scores_bad<G>(sc, (lane & 15) < nvalid);
      block_softmax_pv<G, false>(vbuf, pbufs[warp], lane, nvalid, sc, m[r], l[r], acc[r]);
    }
  }
  if (__any_sync(kFull, bad) && lane == 0 && p.status)
    atomicOr(&p.status[si], kStatusNonFiniteScore);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int jq = warp + 4 * r;
    if (jq >= nq) break;
    const int row = se.row_offset + q0 + jq;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float2 o = make_float2(acc[r][g].x / l[r][g], acc[r][g].y / l[r][g]);
      reinterpret_cast<float2*>(p.out + (static_cast<size_t>(row) * Hq + h * G + g) * D)[lane] = o;
    }
  }
}

// ---------------------------------------------------------------------------
// Attention in the reference's operation order (f32 pools), bit for bit.
// One CTA of 128 threads per (token row, query head): the row's query at
// position qpos attends positions 0..qpos of its sequence's cache, as
// scaled_causal_scores / causal_probabilities / attend_values do for a prompt
// (attention.rs:195-399; masked positions hold f32::MIN, whose exp is 0 and
// which add nothing) and attend_cached_query does for a decoded token
// (attention.rs:677-759). In the fused decode form (every token count 1,
// p.fused) the kernel also does forward_cached_token's append
// (attention.rs:794-810): the new K row rotated at position qpos and the new
// V row come from k_new / v_new, the first query head of each KV group
// stores them into the pool (zeros and kStatusNonFinite when not finite,
// kv_cache.rs:192-197), and every head reads the new row from its inputs,
// never from the pool (another CTA may be writing it):
//   score_j = fold_i fma(q_i, k_j,i) from 0, times (d as f32).sqrt().recip()
//   m = max_j score_j; p_j = exp(score_j - m) (glibc's expf, restated);
//   sum = p_0 + p_1 + ... in order; p_j /= sum           (softmax.rs:26-44)
//   out_d = fold_j fma(v_j,d, p_j, out_d) from 0           (attention.rs:751-756)
// Every thread scores positions (tid, tid + 128, ...); the probabilities live
// in shared memory; thread 0 folds the sum; threads 0-63 each fold one output
// dimension. The value folds are one dependent fma per position, so their
// rows must already be in shared memory: thread 64 starts bulk copies of the
// first kExactStages 16-token V blocks when the CTA starts (they land while
// the scores and the softmax run) and refills each stage once both folding
// warps have read it. A non-finite score or sum flags the sequence
// (softmax.rs:17-22,35-40). Every wait is bounded; on expiry the CTA records
// the timeout, waits (bounded) for its own copies and returns.
// ---------------------------------------------------------------------------
constexpr float kScaleExact = 0.125f;  // (64 as f32).sqrt().recip(), exact
constexpr int kExactThreads = 128;
constexpr int kExactChunk = kBlockTokens * D * 4;  // one 16-token block of V, one head

struct ExactSmem {  // byte offsets in dynamic shared memory
  int stages, kblocks, ring, kst, full, empty, kfull, q, kn, vn, red, ps, total;
};
__host__ __device__ inline ExactSmem exact_smem_layout(int max_ctx, int stages, int kblocks) {
  ExactSmem l;
  l.stages = stages;
  l.kblocks = kblocks;
  l.ring = 0;                                  // stages x 4 KiB, 16-byte aligned
  l.kst = stages * kExactChunk;                // kblocks x 4 KiB: the first K blocks, fused decode
  l.full = l.kst + kblocks * kExactChunk;      // mbarriers
  l.empty = l.full + 8 * stages;
  l.kfull = l.empty + 8 * stages;
  l.q = l.kfull + 16;                          // 64 floats
  l.kn = l.q + D * 4;                          // the new K row (rotated), fused decode
  l.vn = l.kn + D * 4;                         // the new V row
  l.red = l.vn + D * 4;                        // 8 floats + flags
  l.ps = l.red + 64;                           // max_ctx floats
  l.total = l.ps + ((max_ctx + 3) & ~3) * 4;
  return l;
}

constexpr int kExactRoundBlocks = kExactThreads / kBlockTokens;  // K blocks a round: a position a thread

__global__ void __launch_bounds__(kExactThreads) exact_attention_kernel(const PrefillLaunch p,
                                                                        int stages, int kblocks,
                                                                        int kbufs) {
  SLMKV_TL(kTlExact);
  extern __shared__ __align__(128) uint8_t sm_exact[];
  const ExactSmem lay = exact_smem_layout(p.max_ctx, stages, kblocks);
  uint8_t* ring = sm_exact + lay.ring;
  const float* kst = reinterpret_cast<const float*>(sm_exact + lay.kst);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm_exact + lay.full);
  uint64_t* empty = reinterpret_cast<uint64_t*>(sm_exact + lay.empty);
  uint64_t* kfull = reinterpret_cast<uint64_t*>(sm_exact + lay.kfull);
  float* qs = reinterpret_cast<float*>(sm_exact + lay.q);
  float* kns = reinterpret_cast<float*>(sm_exact + lay.kn);
  float* vns = reinterpret_cast<float*>(sm_exact + lay.vn);
  float* red = reinterpret_cast<float*>(sm_exact + lay.red);
  int* flags = reinterpret_cast<int*>(red + 8);  // [0] bad, [1] abort
  float* ps = reinterpret_cast<float*>(sm_exact + lay.ps);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Hq = p.g.q_heads, Hkv = p.g.kv_heads;
  const int r = static_cast<int>(blockIdx.x / Hq), h = static_cast<int>(blockIdx.x % Hq);
  int si = 0;
  if (warp == 0) si = warp_find_seq(p.seqs, p.n_seq, r, lane);
  if (tid == 0) {
    for (int st = 0; st < stages; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], 2);  // one arrival per folding warp
    }
    mbar_init(&kfull[0], 1);
    mbar_init(&kfull[1], 1);
    fence_mbar_init();
    flags[0] = flags[1] = 0;
    reinterpret_cast<int*>(red)[0] = si;
  }
  __syncthreads();
  si = reinterpret_cast<const int*>(red)[0];
  const SeqEntry se = p.seqs[si];
  const int qpos = se.base + (r - se.row_offset);
  const int L = qpos + 1;
  const int nblk = (L + kBlockTokens - 1) / kBlockTokens;
  const int kvh = h / (Hq / Hkv);
  const size_t layer_off = static_cast<size_t>(p.layer) * p.g.layer_elems;
  const float* kb = static_cast<const float*>(p.g.k) + layer_off;
  const float* vb = static_cast<const float*>(p.g.v) + layer_off;
  const int32_t* bt = p.g.block_table + static_cast<size_t>(se.slot) * p.g.max_blocks_per_seq;
  auto chunk_of = [&](const float* base, int b) {
    const int32_t blk = checked_block(p.g, bt[b]);
    return base + (static_cast<size_t>(blk) * Hkv + kvh) * (kBlockTokens * D);
  };
  // Fused decode: the new row is the last block's row n_last - 1; a block
  // holding nothing but the new row is not staged at all.
  const int n_last = L - (nblk - 1) * kBlockTokens;
  const int nload = (p.fused && n_last == 1) ? nblk - 1 : nblk;
  // thread 64: the V ring's producer. In the fused decode form the staged
  // rows are older than this step (and the previous kernel of the stream
  // writes none of the pool), so the first copies go out before the wait.
  int issued = 0;
  auto first_copies = [&]() {
    for (; issued < min(stages, nload); ++issued) {
      mbar_arrive_expect_tx(&full[issued], kExactChunk);
      bulk_load(ring + issued * kExactChunk, chunk_of(vb, issued), kExactChunk, &full[issued]);
    }
  };
  if (tid == 64 && p.fused) first_copies();
  // Fused decode: the K blocks of the older positions are staged too (thread
  // 96, one barrier for all of them; the blocks the V ring stages); the
  // scores read the staged rows. The new row is never read from there (it
  // comes from k_new). With kbufs > 0 (more CTAs than SMs: not every block
  // fits) K passes instead through kbufs buffers of kExactRoundBlocks
  // blocks, a round of 128 positions each (a position a thread), the first
  // rounds requested before the wait and each later one as a buffer frees.
  const int nks = (p.fused && kbufs == 0) ? min(kblocks, nload) : 0;
  const int nrounds = kbufs ? (L + kExactThreads - 1) / kExactThreads : 0;
  auto round_blocks = [&](int rr) { return max(0, min(kExactRoundBlocks, nload - rr * kExactRoundBlocks)); };
  auto issue_round = [&](int rr) {  // thread 96
    const int nb = round_blocks(rr), buf = rr % kbufs;
    if (nb == 0) return;
    mbar_arrive_expect_tx(&kfull[buf], static_cast<uint32_t>(nb) * kExactChunk);
    for (int b = 0; b < nb; ++b)
      bulk_load(const_cast<float*>(kst) + (buf * kExactRoundBlocks + b) * (kExactChunk / 4),
                chunk_of(kb, rr * kExactRoundBlocks + b), kExactChunk, &kfull[buf]);
  };
  int rounds_issued = 0;
  if (tid == 96)
    for (; rounds_issued < min(kbufs, nrounds); ++rounds_issued) issue_round(rounds_issued);
  if (tid == 96 && nks > 0) {
    mbar_arrive_expect_tx(kfull, static_cast<uint32_t>(nks) * kExactChunk);
    for (int b = 0; b < nks; ++b)
      bulk_load(const_cast<float*>(kst) + b * (kExactChunk / 4), chunk_of(kb, b), kExactChunk, kfull);
  }
  // the position's rotation (a constant table) before the wait
  float2 cs = make_float2(0.f, 0.f);
  if (warp < 2 && (p.rotate || p.fused)) cs = p.g.rope[static_cast<size_t>(qpos) * (D / 2) + lane];
  // Launched with programmatic stream serialization in the fused form: the
  // inputs (q, new K/V) are the previous kernel's outputs.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  SLMKV_TL_MARK(kTlExactWaited);
  if (tid == 64 && !p.fused) first_copies();
  if (warp == 0) {
    float2 x = reinterpret_cast<const float2*>(p.q + (static_cast<size_t>(r) * Hq + h) * D)[lane];
    if (p.rotate) x = rope_pair(x, cs);
    reinterpret_cast<float2*>(qs)[lane] = x;
  } else if (warp == 1 && p.fused) {
    // forward_cached_token's append (attention.rs:794-810, kv_cache.rs:182-230)
    const size_t row = (static_cast<size_t>(r) * Hkv + kvh) * D;
    const float2 kx = reinterpret_cast<const float2*>(p.k_new + row)[lane];
    const float2 vx = reinterpret_cast<const float2*>(p.v_new + row)[lane];
    const float2 kr = rope_pair(kx, cs);
    const bool fin = finite2(kx) && finite2(vx);
    reinterpret_cast<float2*>(kns)[lane] = kr;
    reinterpret_cast<float2*>(vns)[lane] = vx;
    if (h % (Hq / Hkv) == 0) {  // one writer per KV head
      const int32_t blk = checked_block(p.g, bt[qpos >> 4]);
      const size_t dst = layer_off + ((static_cast<size_t>(blk) * Hkv + kvh) * kBlockTokens +
                                      (qpos & 15)) * D;
      const float2 z = make_float2(0.f, 0.f);
      reinterpret_cast<float2*>(static_cast<float*>(p.g.k) + dst)[lane] = fin ? kr : z;
      reinterpret_cast<float2*>(static_cast<float*>(p.g.v) + dst)[lane] = fin ? vx : z;
      if (!__all_sync(kFull, fin) && lane == 0 && p.status)
        atomicOr(&p.status[si], kStatusNonFinite);
    }
  }
  __syncthreads();
  // the staged K blocks (a bounded wait; on expiry the scores read the pool)
  int kst_rows = 0;
  if (nks > 0) {
    if (mbar_wait_bounded(&kfull[0], 0)) {
      kst_rows = nks * kBlockTokens;
    } else if (tid == 0) {
      atomicOr(p.g.error, kErrTimeout);
    }
  }
  // ---- scores, two positions per thread at a time ----------------------------
  bool bad = false;
  float mloc = -INFINITY;
  auto key_row = [&](int j) {
    if (p.fused && j == qpos) return reinterpret_cast<const float4*>(kns);
    if (j < kst_rows) return reinterpret_cast<const float4*>(kst + j * D);
    return reinterpret_cast<const float4*>(chunk_of(kb, j >> 4) + (j & 15) * D);
  };
  // K in rounds through the buffers: position rr * 128 + tid in round rr;
  // after a bounded wait that expires the round reads the pool instead, and
  // no later round is requested (flags[1]: the CTA's copies are abandoned)
  for (int rr = 0; rr < nrounds; ++rr) {
    const int nb = round_blocks(rr), buf = rr % kbufs;
    bool staged = false;
    if (nb > 0 && !flags[1]) {
      staged = mbar_wait_bounded(&kfull[buf], static_cast<uint32_t>(rr / kbufs) & 1u);
      if (!staged) {
        flags[1] = 1;
        if (tid == 0) atomicOr(p.g.error, kErrTimeout);
      }
    }
    const int j = rr * kExactThreads + tid;
    if (j < L) {
      const int bj = (j >> 4) - rr * kExactRoundBlocks;
      const float4* k0 = (p.fused && j == qpos) ? reinterpret_cast<const float4*>(kns)
                         : (staged && bj < nb)
                             ? reinterpret_cast<const float4*>(kst + (buf * kExactRoundBlocks + bj) * (kExactChunk / 4) +
                                                               (j & 15) * D)
                             : reinterpret_cast<const float4*>(chunk_of(kb, j >> 4) + (j & 15) * D);
      float a0 = 0.f;
#pragma unroll
      for (int c = 0; c < D / 4; ++c) {
        const float4 q4 = reinterpret_cast<const float4*>(qs)[c];
        const float4 x0 = k0[c];
        a0 = fmaf(q4.x, x0.x, a0);
        a0 = fmaf(q4.y, x0.y, a0);
        a0 = fmaf(q4.z, x0.z, a0);
        a0 = fmaf(q4.w, x0.w, a0);
      }
      const float s0 = __fmul_rn(a0, kScaleExact);
      bad |= !isfinite(s0);
      ps[j] = s0;
      mloc = fmaxf(mloc, s0);
    }
    __syncthreads();  // buffer buf is read
    if (tid == 96 && !flags[1] && rounds_issued < nrounds) issue_round(rounds_issued++);
  }
  for (int j0 = kbufs ? L : tid; j0 < L; j0 += 2 * kExactThreads) {
    const int j1 = j0 + kExactThreads;
    const bool two = j1 < L;
    const int jj1 = two ? j1 : j0;
    const float4* k0 = key_row(j0);
    const float4* k1 = key_row(jj1);
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int c = 0; c < D / 4; ++c) {
      const float4 q4 = reinterpret_cast<const float4*>(qs)[c];
      const float4 x0 = k0[c], x1 = k1[c];
      a0 = fmaf(q4.x, x0.x, a0);
      a1 = fmaf(q4.x, x1.x, a1);
      a0 = fmaf(q4.y, x0.y, a0);
      a1 = fmaf(q4.y, x1.y, a1);
      a0 = fmaf(q4.z, x0.z, a0);
      a1 = fmaf(q4.z, x1.z, a1);
      a0 = fmaf(q4.w, x0.w, a0);
      a1 = fmaf(q4.w, x1.w, a1);
    }
    const float s0 = __fmul_rn(a0, kScaleExact), s1 = __fmul_rn(a1, kScaleExact);
    bad |= !isfinite(s0);
    ps[j0] = s0;
    mloc = fmaxf(mloc, s0);
    if (two) {
      bad |= !isfinite(s1);
      ps[j1] = s1;
      mloc = fmaxf(mloc, s1);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(kFull, mloc, off));
  if (lane == 0) red[warp] = mloc;
  __syncthreads();
  SLMKV_TL_MARK(kTlExactScored);
  const float m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  for (int j = tid; j < L; j += kExactThreads) ps[j] = libm::slm_expf(__fsub_rn(ps[j], m));
  __syncthreads();
  if (tid == 0) {
    float sum = 0.f;
    int j = 0;
    for (; j + 4 <= L; j += 4) {  // ps is 16-byte aligned
      const float4 v = *reinterpret_cast<const float4*>(ps + j);
      sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, v.x), v.y), v.z), v.w);
    }
    for (; j < L; ++j) sum = __fadd_rn(sum, ps[j]);
    red[4] = sum;
  }
  __syncthreads();
  SLMKV_TL_MARK(kTlExactSummed);
  const float sum = red[4];
  bad |= !(isfinite(sum) && sum > 0.f);
  for (int j = tid; j < L; j += kExactThreads) ps[j] = __fdiv_rn(ps[j], sum);
  if (bad) flags[0] = 1;
  __syncthreads();
  SLMKV_TL_MARK(kTlExactSoftmax);
  // ---- values: threads 0-63 fold one dimension each; thread 64 refills -------
  if (tid < D) {
    float o = 0.f;
    for (int b = 0; b < nload; ++b) {
      const int st = b % stages;
      if (!mbar_wait_bounded(&full[st], static_cast<uint32_t>(b / stages) & 1u)) {
        flags[1] = 1;
        atomicOr(p.g.error, kErrTimeout);
        break;
      }
      if (flags[1]) break;
      const float* vr = reinterpret_cast<const float*>(ring + st * kExactChunk) + tid;
      // the fused form's new row comes from its input, not from the pool
      const int n = min(kBlockTokens, L - b * kBlockTokens) - ((p.fused && b == nblk - 1) ? 1 : 0);
      const float* pb = ps + b * kBlockTokens;
      if (n == kBlockTokens) {
#pragma unroll
        for (int t = 0; t < kBlockTokens; ++t) o = fmaf(vr[t * D], pb[t], o);
      } else {
        for (int t = 0; t < n; ++t) o = fmaf(vr[t * D], pb[t], o);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (p.fused && !flags[1]) o = fmaf(vns[tid], ps[qpos], o);
    p.out[(static_cast<size_t>(r) * Hq + h) * D + tid] = o;
    SLMKV_TL_MARK(kTlExactFolded);
  } else if (tid == 64) {
    for (; issued < nload; ++issued) {
      const int st = issued % stages;
      if (flags[1] ||
          !mbar_wait_bounded(&empty[st], static_cast<uint32_t>(issued / stages - 1) & 1u)) {
        flags[1] = 1;
        atomicOr(p.g.error, kErrTimeout);
        break;
      }
      mbar_arrive_expect_tx(&full[st], kExactChunk);
      bulk_load(ring + st * kExactChunk, chunk_of(vb, issued), kExactChunk, &full[st]);
    }
    // every copy issued lands before the CTA's shared memory is released
    for (int b = max(0, issued - stages); b < issued; ++b)
      mbar_wait_bounded(&full[b % stages], static_cast<uint32_t>(b / stages) & 1u);
    if (nks > 0 && kst_rows == 0) mbar_wait_bounded(&kfull[0], 0);  // the K copies, after a timeout
  } else if (tid == 96 && kbufs > 0) {
    // K rounds requested and not consumed (after an abandoned round) land
    // before the CTA's shared memory is released
    for (int rr = max(0, rounds_issued - kbufs); rr < rounds_issued; ++rr)
      if (round_blocks(rr) > 0) mbar_wait_bounded(&kfull[rr % kbufs], static_cast<uint32_t>(rr / kbufs) & 1u);
  }
  __syncthreads();
  if (tid == 0 && flags[0] && p.status) atomicOr(&p.status[si], kStatusNonFiniteScore);
}

// ---------------------------------------------------------------------------
// Block-table writes, then copy-on-write block copies (all layers, K and V).
// ---------------------------------------------------------------------------
__global__ void apply_updates_kernel(const PoolGeom g, const TableUpdate* __restrict__ up,
                                     int32_t nu, const CopyJob* __restrict__ cp, int32_t nc) {
  SLMKV_TL(kTlApply);
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = tid; i < nu; i += stride) {
    const TableUpdate u = up[i];
    g.block_table[static_cast<size_t>(u.slot) * g.max_blocks_per_seq + u.index] = u.block;
  }
  const int esz = g.bf16 ? 2 : 4;
  const int64_t chunk16 = static_cast<int64_t>(g.kv_heads) * kBlockTokens * D * esz / 16;
  const int64_t per_job = chunk16 * g.num_layers * 2;
  for (int64_t i = tid; i < per_job * nc; i += stride) {
    const int64_t job = i / per_job;
    int64_t r = i - job * per_job;
    const int pool = static_cast<int>(r / (chunk16 * g.num_layers));
    r -= static_cast<int64_t>(pool) * chunk16 * g.num_layers;
    const int layer = static_cast<int>(r / chunk16);
    const int64_t e = r - static_cast<int64_t>(layer) * chunk16;
    const int32_t src = checked_block(g, cp[job].src), dst = checked_block(g, cp[job].dst);
    uint8_t* base = static_cast<uint8_t*>(pool ? g.v : g.k) +
                    static_cast<size_t>(layer) * g.layer_elems * esz;
    const uint4* s = reinterpret_cast<const uint4*>(base + static_cast<size_t>(src) * chunk16 * 16);
    uint4* d = reinterpret_cast<uint4*>(base + static_cast<size_t>(dst) * chunk16 * 16);
    d[e] = s[e];
  }
}

}  // namespace

cudaError_t launch_decode(const StreamDecodeLaunch& p, cudaStream_t s) {
  const int G = p.g.q_heads / p.g.kv_heads;
  if (p.g.bf16) {
    switch (G) {
      case 1: return launch_decode_t<1, 1>(p, s);
      case 2: return launch_decode_t<1, 2>(p, s);
      case 4: return launch_decode_t<1, 4>(p, s);
      case 8: return launch_decode_t<1, 8>(p, s);
    }
  } else {
    switch (G) {
      case 1: return launch_decode_t<0, 1>(p, s);
      case 2: return launch_decode_t<0, 2>(p, s);
      case 4: return launch_decode_t<0, 4>(p, s);
      case 8: return launch_decode_t<0, 8>(p, s);
    }
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_append(const AppendLaunch& p, cudaStream_t s) {
  const int64_t rows = static_cast<int64_t>(p.total_tokens) * p.g.kv_heads;
  if (rows <= 0) return cudaSuccess;
  const int64_t blocks = (rows + kAppendRows - 1) / kAppendRows;
  if (p.g.bf16) append_kernel<1><<<static_cast<unsigned>(blocks), 256, 0, s>>>(p);
  else append_kernel<0><<<static_cast<unsigned>(blocks), 256, 0, s>>>(p);
  return cudaGetLastError();
}

// V ring depth: a few rows (batch-1 decode) run one CTA per SM or less, and
// each CTA's value fold waits on its own copies, so the ring is deep (16
// blocks in flight from the CTA's start); many rows keep several CTAs per SM
// busy, which hides the copies, so the ring is shallow and more CTAs fit.
int exact_attention_stages(int32_t max_ctx, int64_t items) {
  const int want = items <= 2 * 148 ? 16 : 4;
  for (int st = want; st >= 2; --st)
    if (exact_smem_layout(max_ctx, st, 0).total <= 227 * 1024) return st;
  return 0;
}
// Fused decode with at most one CTA an SM: the K blocks staged before the
// wait, as many as the shared memory left holds (with more CTAs, staging
// would leave room for one CTA an SM and need a second wave)
int exact_attention_kblocks(const PrefillLaunch& p, int stages, int64_t items) {
  if (!p.fused || items > 148) return 0;
  const int want = (p.max_ctx + kBlockTokens - 1) / kBlockTokens;
  const int room = (227 * 1024 - exact_smem_layout(p.max_ctx, stages, 0).total) / kExactChunk;
  return max(0, min(want, room));
}
// Fused decode with more CTAs than SMs: K rounds through two buffers (one
// CTA in two SMs' worth of rows: two CTAs an SM) or one (more), the V ring 8
// or 4 deep; none when the rows' probabilities leave no room.
struct ExactShape {
  int stages, kblocks, kbufs;
};
ExactShape exact_attention_shape(const PrefillLaunch& p, int64_t items) {
  ExactShape sh{exact_attention_stages(p.max_ctx, items), 0, 0};
  if (sh.stages == 0) return sh;
  if (p.fused && items > 148) {
    const ExactShape r{items <= 2 * 148 ? 8 : 4, 0, items <= 2 * 148 ? 2 : 1};
    if (exact_smem_layout(p.max_ctx, r.stages, r.kbufs * kExactRoundBlocks).total <= 100 * 1024)
      return ExactShape{r.stages, r.kbufs * kExactRoundBlocks, r.kbufs};
    return sh;
  }
  sh.kblocks = exact_attention_kblocks(p, sh.stages, items);
  return sh;
}

cudaError_t launch_exact_attention(const PrefillLaunch& p0, cudaStream_t s) {
  if (p0.n_seq <= 0 || p0.total_tokens <= 0) return cudaSuccess;
  if (p0.g.bf16) return cudaErrorInvalidValue;
  PrefillLaunch p = p0;
  p.max_ctx = (p.max_ctx + 3) & ~3;
  const int64_t items = static_cast<int64_t>(p.total_tokens) * p.g.q_heads;
  const ExactShape sh = exact_attention_shape(p, items);
  if (sh.stages == 0) return cudaErrorInvalidValue;
  const int stages = sh.stages, kblocks = sh.kblocks;
  const int smem = exact_smem_layout(p.max_ctx, stages, kblocks).total;
  cudaError_t e = cudaFuncSetAttribute(exact_attention_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(items));
  cfg.blockDim = dim3(kExactThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.fused ? 1 : 0;  // the fused decode chains onto the q/k/v kernel
  return cudaLaunchKernelEx(&cfg, exact_attention_kernel, p, stages, kblocks, sh.kbufs);
}

cudaError_t launch_gather(const GatherLaunch& p, cudaStream_t s) {
  const int64_t rows = static_cast<int64_t>(p.length) * p.g.kv_heads;
  if (rows <= 0) return cudaSuccess;
  const int threads = 256;
  const int64_t blocks = (rows * 16 + threads - 1) / threads;
  if (p.g.bf16) gather_kernel<1><<<static_cast<unsigned>(blocks), threads, 0, s>>>(p);
  else gather_kernel<0><<<static_cast<unsigned>(blocks), threads, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_prefill(const PrefillLaunch& p, cudaStream_t s) {
  if (p.n_seq <= 0 || p.max_count <= 0) return cudaSuccess;
  if (prefill_tc_supported(p)) return launch_prefill_tc(p, s);
  const dim3 grid((p.max_count + kBlockTokens - 1) / kBlockTokens, p.n_seq, p.g.kv_heads);
  const int G = p.g.q_heads / p.g.kv_heads;
#define SLMKV_PREFILL(B, GG) prefill_kernel<B, GG><<<grid, 128, 0, s>>>(p)
  if (p.g.bf16) {
    switch (G) {
      case 1: SLMKV_PREFILL(1, 1); break;
      case 2: SLMKV_PREFILL(1, 2); break;
      case 4: SLMKV_PREFILL(1, 4); break;
      default: return cudaErrorInvalidValue;
    }
  } else {
    switch (G) {
      case 1: SLMKV_PREFILL(0, 1); break;
      case 2: SLMKV_PREFILL(0, 2); break;
      case 4: SLMKV_PREFILL(0, 4); break;
      default: return cudaErrorInvalidValue;
    }
  }
#undef SLMKV_PREFILL
  return cudaGetLastError();
}

cudaError_t launch_apply_updates(const PoolGeom& g, const TableUpdate* updates, int32_t n_updates,
                                 const CopyJob* copies, int32_t n_copies, cudaStream_t s) {
  if (n_updates <= 0 && n_copies <= 0) return cudaSuccess;
  const int threads = 256;
  const int64_t esz = g.bf16 ? 2 : 4;
  const int64_t work =
      n_updates + static_cast<int64_t>(n_copies) * g.num_layers * 2 * g.kv_heads * kBlockTokens * D *
                      esz / 16;
  int64_t blocks = (work + threads - 1) / threads;
  if (blocks > 4096) blocks = 4096;
  if (blocks < 1) blocks = 1;
  apply_updates_kernel<<<static_cast<unsigned>(blocks), threads, 0, s>>>(g, updates, n_updates,
                                                                          copies, n_copies);
  return cudaGetLastError();
}

SLMKV_TL_SETTER(timeline_set_kernels)

}  // namespace slmkv
