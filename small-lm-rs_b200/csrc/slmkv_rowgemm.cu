// Few-row projections on the tensor cores (tcgen05): y[rows, cols] = x[rows, K]
// . w[K, cols] for the model step's q/k/v, output, gate/up and down
// projections when a step has a few hundred token rows or fewer (decode
// batches), where a library GEMM runs tiny grids and does not stream the
// weights at HBM speed.
//
// The product is computed transposed, D^T = w^T x^T: the weights are the MMA's
// A operand (M = 128 output columns a CTA, read MN-major straight from their
// [in][out] layout: two 64-column TMA boxes a stage), the token rows its B
// operand (N = 16, 64 or 128 rows, K-major), so a handful of rows costs no
// padding and the fp32 accumulator sits in TMEM with one output column per
// lane. K streams through a ring of TMA stages, 64 input features a stage;
// when the output tiles alone cannot fill the SMs, K is split across the CTAs
// of a thread-block cluster (up to 8), which add their partial sums in split
// order (deterministic) over distributed shared memory, each CTA for its
// share of the rows, and run the epilogue:
//   QKV   q | k | v columns to their three outputs
//   O     onto the residual stream (transformer.rs add_residual_in_place)
//   GU    gate and up tiles side by side (lanes 0-63 gate, 64-127 up of the
//         same 64 columns), SiTU-GLU (situ_glu.rs:101-107,131-138:
//         b_g tanh(g / b_g) sigmoid(g) * b_u tanh(u / b_u)), h as bf16
//   Down  onto the residual stream
//   Head  the vocabulary logits (fp32, plain stores): the fp32 tied head as
//         one bf16 GEMM over K = 3H, the rows split x = xh + xl and the
//         weights w = wh + wl (both bf16), summing xh.wh + xl.wh + xh.wl:
//         K chunk 2c is xh_c . wh_c and 2c + 1 xl_c . wh_c (the same weight
//         box twice in a row, the second read from L2), then xh . wl; the
//         weights are [wh; wl], [2H][V]
// The RMSNorm between a residual update and the next projection
// (rmsnorm.rs:80-91: x * inv_rms * g) needs no kernel of its own: O and Down
// also write bf16(x * g) and each row's square sum over their tile, and QKV
// and GU multiply each row's reduced sums by inv_rms, which they compute from
// those square sums (the same product up to where the bf16 rounding falls).
// Operands are bf16 with fp32 accumulation (linear.rs:44-107 up to the
// accumulation order). Launched with programmatic stream serialization: the
// first stages' weight boxes are requested before the previous kernel
// completes; everything that reads or writes activations waits for it.
// Every mbarrier wait is bounded (about 1 s): on expiry the CTA sets the
// context's timeout bit, waits (bounded) for its own copies in flight, still
// takes part in the cluster barriers and returns. No TMA multicast.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdint>

#include "slmkv_internal.h"

namespace slmkv {
namespace {

constexpr int kRgThreads = 128;
constexpr int kRgTileM = 128;  // output columns a CTA
constexpr int kRgChunk = 64;   // input features a stage
constexpr int kRgABytes = kRgTileM * kRgChunk * 2;  // 16 KiB: two 64 x 64 boxes
constexpr unsigned long long kRgWaitNs = 1000000000ull;
constexpr int kRgSpinsMax = 1 << 26;
constexpr int kRgMaxSplits = 8;  // K splits a tile: one thread-block cluster (portable size)

constexpr int rg_ctas_per_sm(int rt) { return rt <= 16 ? 2 : 1; }  // shared-memory bound
template <int RT>
struct RgCfg {
  static constexpr int kBBytes = RT * kRgChunk * 2;  // RT rows of 128 B
  static constexpr int kStageBytes = kRgABytes + kBBytes;
  // 16 rows: 6 stages (108 KiB), two CTAs an SM; more rows: one CTA an SM
  static constexpr int kStages = RT <= 16 ? 6 : RT <= 64 ? 8 : 6;
  static constexpr int kTmemCols = RT < 32 ? 32 : RT;
  static constexpr int kSmem = kStages * kStageBytes + 1024;  // + alignment slack
  static_assert(RT * kRgTileM * 4 <= kStages * kStageBytes, "partial tile fits in the stages");
};

__device__ __forceinline__ uint32_t rg_su32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long rg_timer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool rg_try(uint32_t bar, uint32_t parity) {
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
// true once the phase with this parity has completed; false after ~1 s
__device__ __forceinline__ bool rg_wait(uint32_t bar, uint32_t parity) {
  if (rg_try(bar, parity)) return true;
  const unsigned long long t0 = rg_timer();
  for (int i = 0; i < kRgSpinsMax; ++i) {
    if (rg_try(bar, parity)) return true;
    if ((i & 255) == 255 && rg_timer() - t0 > kRgWaitNs) return false;
  }
  return false;
}
__device__ __forceinline__ void rg_tma(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// shared-memory matrix descriptor, 128-byte swizzle (start, leading and stride
// byte offsets in 16-byte units, sm_100 version field)
__device__ __forceinline__ uint64_t rg_desc(uint32_t addr, uint32_t lbo16, uint32_t sbo16) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(lbo16 & 0x3FFFu) << 16) |
         (static_cast<uint64_t>(sbo16 & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// instruction descriptor, kind::f16: f32 D, bf16 A and B, A MN-major, B K-major
constexpr uint32_t rg_idesc(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}
__device__ __forceinline__ void rg_mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(id), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void rg_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void rg_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void rg_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <int MODE, int RT>
__global__ void __launch_bounds__(kRgThreads, 1) row_gemm_kernel(const __grid_constant__ RowGemmLaunch p) {
  SLMKV_TL(kTlRowGemm + MODE);
  using Cfg = RgCfg<RT>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t rg_smem_raw[];
  __shared__ __align__(8) uint64_t bars[2 * S + 1];  // full[S], empty[S], done
  __shared__ uint32_t tmem_slot;
  __shared__ int32_t aborted;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // The next kernel may be scheduled as soon as every CTA of this grid is
  // resident: before its own wait it only requests weights, and it waits for
  // this grid's completion before it touches activations.
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(rg_smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = rg_su32(sm);
  const uint32_t full0 = rg_su32(&bars[0]), empty0 = rg_su32(&bars[S]), done = rg_su32(&bars[2 * S]);
  const int col_tile = blockIdx.x, row_tile = blockIdx.y, split = blockIdx.z;
  const int ch0 = split * p.chunks_per_split;
  const int nch = min(p.nchunks, ch0 + p.chunks_per_split) - ch0;  // >= 1 by construction
  if (tid == 0) {
    for (int s = 0; s < 2 * S + 1; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(rg_su32(&bars[s])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    aborted = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(rg_su32(&tmem_slot)),
                 "r"(Cfg::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;
  auto raise_abort = [&]() {
    atomicExch(&aborted, 1);
    atomicOr(p.err, kErrTimeout);
  };
  // A boxes: output columns (QKV, O, Down: 128 adjacent; GU: 64 gate and the
  // 64 up columns I later)
  const int xa0 = MODE == kRowGU ? kRgChunk * col_tile : kRgTileM * col_tile;
  const int xa1 = MODE == kRowGU ? p.I + kRgChunk * col_tile : xa0 + kRgChunk;
  const int yb = row_tile * RT;
  // the weight row of K row ky (the head's interleaved order; others: ky)
  auto a_row = [&](int ky) {
    if (MODE != kRowHead) return ky;
    return ky < 2 * p.H ? (ky >> 7) << 6 : ky - p.H;
  };
  auto stage_a = [&](int s) { return sbase + s * Cfg::kStageBytes; };
  auto stage_b = [&](int s) { return sbase + s * Cfg::kStageBytes + kRgABytes; };

  if (warp == 0) {
    if (lane == 0) {
      // ---- producer: weight boxes of the first stages, the wait, then the rows ----
      const int pre = min(nch, S);
      for (int i = 0; i < pre; ++i) {
        const uint32_t fb = full0 + 8 * i;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fb),
                     "r"(Cfg::kStageBytes)
                     : "memory");
        const int ky = (ch0 + i) * kRgChunk, ay = a_row(ky);
        rg_tma(stage_a(i), &p.tmap_w, xa0, ay, fb);
        rg_tma(stage_a(i) + kRgABytes / 2, &p.tmap_w, xa1, ay, fb);
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      SLMKV_TL_MARK(kTlRowGemmWaited + MODE);
      for (int i = 0; i < pre; ++i) rg_tma(stage_b(i), &p.tmap_x, (ch0 + i) * kRgChunk, yb, full0 + 8 * i);
      int issued = pre;
      for (int i = pre; i < nch; ++i) {
        const int s = i % S;
        if (!rg_wait(empty0 + 8 * s, ((i / S) - 1) & 1)) {
          raise_abort();
          break;
        }
        const uint32_t fb = full0 + 8 * s;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fb),
                     "r"(Cfg::kStageBytes)
                     : "memory");
        const int ky = (ch0 + i) * kRgChunk, ay = a_row(ky);
        rg_tma(stage_a(s), &p.tmap_w, xa0, ay, fb);
        rg_tma(stage_a(s) + kRgABytes / 2, &p.tmap_w, xa1, ay, fb);
        rg_tma(stage_b(s), &p.tmap_x, ky, yb, fb);
        issued = i + 1;
      }
      // on an abort, the copies in flight land before the CTA goes on
      if (issued < nch)
        for (int i = max(0, issued - S); i < issued; ++i) rg_wait(full0 + 8 * (i % S), (i / S) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issue: D[128 cols, RT rows] += W^T[128, 64] x^T[64, RT] per stage ----
      constexpr uint32_t id = rg_idesc(kRgTileM, RT);
      for (int i = 0; i < nch; ++i) {
        const int s = i % S;
        if (!rg_wait(full0 + 8 * s, (i / S) & 1)) {
          raise_abort();
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (int kk = 0; kk < kRgChunk / 16; ++kk)
          rg_mma(tmem, rg_desc(stage_a(s) + 2048 * kk, (kRgABytes / 2) >> 4, 64),
                 rg_desc(stage_b(s) + 32 * kk, 1, 64), id, (i > 0 || kk > 0) ? 1u : 0u);
        rg_commit(empty0 + 8 * s);
      }
      rg_commit(done);  // arrives when every MMA issued above has completed
    }
    __syncwarp();
  }

  // ---- epilogue ----
  // Each CTA moves its accumulator (one tile column a thread, its TMEM lane)
  // to shared memory; the K splits of a tile are one thread-block cluster, so
  // after a cluster barrier CTA c reduces rows c, c + S, ... of the tile,
  // reading every split's partial from its shared memory (DSMEM) and adding
  // them in split order, and writes those rows. One split: the same, S = 1.
  const int m = warp * 32 + lane;
  const int r0 = row_tile * RT, nr = min(RT, p.rows - r0);
  constexpr bool kResidual = MODE == kRowO || MODE == kRowDown;
  constexpr bool kNormed = MODE == kRowQKV || MODE == kRowGU;
  __shared__ float inv_s[kNormed ? RT : 1];         // the deferred RMSNorm's 1 / rms per row
  __shared__ float red_s[kResidual ? 4 : 1][RT];    // per-warp square sums per row
  float gn = 0.f;  // the next norm's scale for this thread's column (a weight)
  if (kResidual && p.norm_next != nullptr && kRgTileM * col_tile + m < p.ncols)
    gn = p.norm_next[kRgTileM * col_tile + m];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (kResidual && warp >= 2) {
    // the residual rows this CTA updates (rows split, split + S, ...; 128
    // columns = four 128-byte lines a row) into L1 while the MMAs run
    const int splits = gridDim.z;
    const int nrow = nr > split ? (nr - split + splits - 1) / splits : 0;
    for (int i = tid - 64; i < 4 * nrow; i += 64) {
      const int r = split + (i >> 2) * splits;
      const int c = kRgTileM * col_tile + 32 * (i & 3);
      if (c < p.ncols)
        asm volatile("prefetch.global.L1 [%0];" ::"l"(p.y0 + static_cast<size_t>(r0 + r) * p.ncols + c));
    }
  }
  if (kNormed && p.ssq_in != nullptr && warp >= 2) {
    // rmsnorm.rs:80-91's 1 / sqrt(mean square + eps), the square sum from
    // the previous projection's tiles; the MMAs may still be running
    for (int r = tid - 64; r < nr; r += 64) {
      const float* sr = p.ssq_in + static_cast<size_t>(r0 + r) * p.ssq_ld;
      float t = 0.f;
#pragma unroll 4
      for (int i = 0; i < p.ssq_ld; ++i) t += sr[i];
      inv_s[r] = 1.f / sqrtf(__fdiv_rn(t, static_cast<float>(p.H)) + p.eps);
    }
  }
  bool ok = true;
  if (lane == 0) ok = rg_wait(done, 0);
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  if (!ok && lane == 0) raise_abort();
  if (warp == 0) SLMKV_TL_MARK(kTlRowGemmMmaDone + MODE);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  __syncthreads();
  const bool run = *reinterpret_cast<volatile int32_t*>(&aborted) == 0;  // CTA-uniform
  float* part = reinterpret_cast<float*>(sm);  // [RT][128]: the stages are idle, every MMA completed
  if (run) {
    const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll 1
    for (int g = 0; g < RT / 16; ++g) {
      float v[16];
      rg_ld16(taddr + 16 * g, v);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int j = 0; j < 16; ++j) part[(16 * g + j) * kRgTileM + m] = v[j];
    }
  }
  rg_cluster_sync();  // every CTA of the cluster arrives, an aborted one too
  if (warp == 0) SLMKV_TL_MARK(kTlRowGemmPartials + MODE);
  const int splits = gridDim.z;
  const uint32_t part_addr = rg_su32(part);
  uint32_t peer[kRgMaxSplits];
#pragma unroll
  for (int sp = 0; sp < kRgMaxSplits; ++sp) {
    uint32_t a = 0;
    if (sp < splits) asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(part_addr), "r"(sp));
    peer[sp] = a;
  }
  // row r, tile column c summed over the splits in split order: every
  // split's value is requested first (the loads depend only on the addresses
  // mapped after the barrier), then added in order
  auto reduced = [&](int r, int c) {
    float x[kRgMaxSplits];
#pragma unroll
    for (int sp = 0; sp < kRgMaxSplits; ++sp) {
      x[sp] = 0.f;
      if (sp < splits)
        asm("ld.shared::cluster.f32 %0, [%1];" : "=f"(x[sp]) : "r"(peer[sp] + 4u * static_cast<uint32_t>(r * kRgTileM + c)));
    }
    float t = 0.f;
#pragma unroll
    for (int sp = 0; sp < kRgMaxSplits; ++sp)
      if (sp < splits) t += x[sp];
    return t;
  };
  if (run) {
    if (MODE == kRowGU) {
      // every thread: tile column c (gate c, up c + 64) for every other of
      // this CTA's rows, so all 128 threads share the SiTU-GLU work
      const int c = m & 63, half = m >> 6;
      const int col = kRgChunk * col_tile + c;
      if (col < p.I) {
        for (int r = split + half * splits; r < nr; r += 2 * splits) {
          float gv = reduced(r, c), u = reduced(r, c + 64);
          if (p.ssq_in != nullptr) {
            gv = __fmul_rn(gv, inv_s[r]);
            u = __fmul_rn(u, inv_s[r]);
          }
          // CUDA's tanhf and exp: this path is held to a tolerance (its
          // accumulation order is the tensor cores'), and glibc's branchy
          // expm1f-based tanhf restated (the exact-order kernels' form)
          // diverges across the lanes and took 3 us more a launch
          const float ga = p.beta_gate * tanhf(gv * (1.f / p.beta_gate)) * __fdividef(1.f, 1.f + __expf(-gv));
          const float ua = p.beta_up * tanhf(u * (1.f / p.beta_up));
          static_cast<__nv_bfloat16*>(p.h)[static_cast<size_t>(r0 + r) * p.I + col] =
              __float2bfloat16_rn(__fmul_rn(ga, ua));
        }
      }
    } else if (MODE == kRowHead) {
      const int col = kRgTileM * col_tile + m;
      if (col < p.ncols)
        for (int r = split; r < nr; r += splits) p.y0[static_cast<size_t>(r0 + r) * p.ncols + col] = reduced(r, m);
    } else if (MODE == kRowQKV) {
      const int col = kRgTileM * col_tile + m;
      if (col < p.ncols) {
        for (int r = split; r < nr; r += splits) {
          float v = reduced(r, m);
          if (p.ssq_in != nullptr) v = __fmul_rn(v, inv_s[r]);
          const size_t row = static_cast<size_t>(r0 + r);
          if (col < p.H) p.y0[row * p.H + col] = v;
          else if (col < p.H + p.KV) p.y1[row * p.KV + col - p.H] = v;
          else p.y2[row * p.KV + col - p.H - p.KV] = v;
        }
      }
    } else {
      // onto the residual stream; with norm_next, also the next projection's
      // operand and the tile's square sum of each row (every thread takes
      // part in the per-row reductions)
      const int col = kRgTileM * col_tile + m;
      const bool has = col < p.ncols, norm = p.norm_next != nullptr;
      int it = 0;
      for (int r = split; r < nr; r += splits, ++it) {
        float y = 0.f;
        const size_t row = static_cast<size_t>(r0 + r);
        if (has) {
          float* yp = p.y0 + row * p.ncols + col;
          y = __fadd_rn(*yp, reduced(r, m));
          *yp = y;
          if (norm)
            static_cast<__nv_bfloat16*>(p.xg)[row * p.ncols + col] = __float2bfloat16_rn(__fmul_rn(y, gn));
        }
        if (norm) {
          float sq = __fmul_rn(y, y);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
          if (lane == 0) red_s[warp][it] = sq;
        }
      }
      if (norm) {
        __syncthreads();
        for (int i = tid; i < it; i += kRgThreads)
          p.ssq[static_cast<size_t>(r0 + split + i * splits) * p.ssq_ld + col_tile] =
              ((red_s[0][i] + red_s[1][i]) + red_s[2][i]) + red_s[3][i];
      }
    }
  }
  if (warp == 0) SLMKV_TL_MARK(kTlRowGemmStored + MODE);
  rg_cluster_sync();  // no CTA leaves (with its shared memory) while another may read it
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::kTmemCols)
                 : "memory");
}

PFN_cuTensorMapEncodeTiled_v12000 rg_encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }();
  return encode;
}

template <int MODE, int RT>
cudaError_t launch_rt(const RowGemmLaunch& p, dim3 grid, cudaStream_t s) {
  static unsigned long long configured = 0;  // one bit per device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 64 && !(configured & (1ull << dev))) {
    e = cudaFuncSetAttribute(row_gemm_kernel<MODE, RT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             RgCfg<RT>::kSmem);
    if (e != cudaSuccess) return e;
    configured |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kRgThreads);
  cfg.dynamicSmemBytes = RgCfg<RT>::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;  // the K splits of a tile
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = grid.z;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, row_gemm_kernel<MODE, RT>, p);
}

template <int MODE>
cudaError_t launch_mode(const RowGemmLaunch& p, int rt, dim3 grid, cudaStream_t s) {
  if (rt == 16) return launch_rt<MODE, 16>(p, grid, s);
  if (rt == 64) return launch_rt<MODE, 64>(p, grid, s);
  return launch_rt<MODE, 128>(p, grid, s);
}

}  // namespace

RowGemmPlan plan_row_gemm(int mode, int32_t rows, int32_t K, int32_t ncols, int32_t sms) {
  RowGemmPlan q{};
  q.rt = rows <= 16 ? 16 : rows <= 64 ? 64 : 128;
  q.row_tiles = (rows + q.rt - 1) / q.rt;
  q.col_tiles = mode == kRowGU ? (ncols + kRgChunk - 1) / kRgChunk : (ncols + kRgTileM - 1) / kRgTileM;
  q.nchunks = (K + kRgChunk - 1) / kRgChunk;
  // split K so that the CTAs fill the SMs in one wave: at most the resident
  // CTAs, at most kRgMaxSplits splits (one cluster)
  const int tiles = q.col_tiles * q.row_tiles;
  const int resident = sms * rg_ctas_per_sm(q.rt);
  const int want = std::min(kRgMaxSplits, std::max(1, resident / tiles));
  q.chunks_per_split = (q.nchunks + want - 1) / want;
  q.splits = (q.nchunks + q.chunks_per_split - 1) / q.chunks_per_split;
  return q;
}

cudaError_t encode_row_gemm_map(CUtensorMap* map, const void* base, int32_t inner, int32_t outer,
                                int32_t box_inner, int32_t box_outer) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = rg_encoder();
  if (!encode) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                            box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_row_gemm(int mode, RowGemmLaunch p, const RowGemmPlan& q, cudaStream_t s) {
  // the rows' map: [rows][K] bf16, boxes of 64 features x rt rows (rows past
  // the end read as zeros)
  cudaError_t e = encode_row_gemm_map(&p.tmap_x, p.x, p.K, p.rows, kRgChunk, q.rt);
  if (e != cudaSuccess) return e;
  p.nchunks = q.nchunks;
  p.chunks_per_split = q.chunks_per_split;
  const dim3 grid(q.col_tiles, q.row_tiles, q.splits);
  switch (mode) {
    case kRowQKV: return launch_mode<kRowQKV>(p, q.rt, grid, s);
    case kRowO: return launch_mode<kRowO>(p, q.rt, grid, s);
    case kRowGU: return launch_mode<kRowGU>(p, q.rt, grid, s);
    case kRowHead: return launch_mode<kRowHead>(p, q.rt, grid, s);
    default: return launch_mode<kRowDown>(p, q.rt, grid, s);
  }
}

SLMKV_TL_SETTER(timeline_set_rowgemm)

}  // namespace slmkv
