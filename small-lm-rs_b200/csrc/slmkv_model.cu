// Full-model steps around the KV path: SmallLMModel's cached decode
// (model.rs:342-397) and prompt prefill (model.rs:297-330) with the
// transformer block of transformer.rs:221-292, on the device.
//
// Per layer: RMSNorm (rmsnorm.rs:80-91) into bf16 rows -> q/k/v projections
// -> the batch's cache step (RoPE, append, attention: slmkv_kernels.cu) ->
// output projection accumulated onto the residual -> RMSNorm -> gate/up
// projections (one GEMM over the concatenated [gate; up] matrix) -> SiTU-GLU
// activations (situ_glu.rs:59-70) into bf16 rows -> down projection
// accumulated onto the residual. Then the final RMSNorm and the tied fp32
// vocabulary projection (model.rs:193-227), and the first maximal logit
// (greedy.rs argmax_finite).
//
// Projections follow linear.rs:44-107: both operands rounded to bf16 (the
// weights once, at upload; the activations where they are produced or
// staged, round-to-nearest-even as linear.rs:14-23), products exact in fp32,
// fp32 accumulation. Up to kFusedRows token rows (decode steps, short
// prompts) they are this file's fused kernels, whose every output is the
// reference's own in-order fold, with the RMSNorm, the attention output's
// rounding, SiTU-GLU and the residual add fused in (5 launches a layer with
// the cache step). Beyond that (long prefills) they are tensor-core GEMMs in
// cuBLAS (bf16 inputs, CUBLAS_COMPUTE_32F; the residual add as beta = 1),
// whose accumulation order differs. The vocabulary projection is an fp32
// SGEMM (no TF32: the handle keeps the default math mode), as
// linear.rs:119-152.
#include <cublas_v2.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "slmkv.h"
#include "slmkv_internal.h"
#include "slmkv_libm.h"

namespace slmkv {
namespace {

// Programmatic dependent launch. The single-row steps are chains of short
// kernels; launched with programmatic stream serialization, a kernel's CTAs
// start while the previous kernel finishes and run what depends on no
// earlier kernel (the immutable weights' first copies). Every such kernel
// calls this before it reads or writes anything another kernel of the
// stream touches: it returns once the previous kernel has completed and its
// memory is visible, and only then lets the next kernel launch. Without the
// launch attribute both instructions are no-ops.
__device__ __forceinline__ void wait_previous_kernel() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... Params, typename... Args>
cudaError_t launch_chained(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                           Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// embedding.rs:15-56: row r <- table[ids[r]]; an id outside the vocabulary
// sets the context's error bit and reads row 0 (the step then fails).
__global__ void embed_kernel(const int32_t* __restrict__ ids, const float* __restrict__ table,
                             int32_t vocab, int32_t hidden, float* __restrict__ x,
                             int32_t* __restrict__ err) {
  SLMKV_TL(kTlEmbed);
  wait_previous_kernel();
  const int r = blockIdx.x;
  int32_t id = ids[r];
  if (static_cast<uint32_t>(id) >= static_cast<uint32_t>(vocab)) {
    if (threadIdx.x == 0) atomicOr(err, kErrBadToken);
    id = 0;
  }
  const float4* src = reinterpret_cast<const float4*>(table + static_cast<size_t>(id) * hidden);
  float4* dst = reinterpret_cast<float4*>(x + static_cast<size_t>(r) * hidden);
  for (int i = threadIdx.x; i < hidden / 4; i += blockDim.x) dst[i] = src[i];
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// rmsnorm.rs:80-91, one CTA per row: square sum (fma; per thread, then a
// warp and a CTA tree in fixed order), inverse RMS 1 / sqrt(s / width + eps),
// out = x * inv * scale (two products, in that order). The row stays in
// registers (all its loads in flight at once). Output rows are bf16 (the
// next projection's rounded operand) or fp32 (the vocabulary projection's).
// With `seqs`, output row i normalises the last token row of sequence i (the
// prefill's final positions).
constexpr int kNormThreads = 256;
constexpr int kNormVec = 8;  // float4s a thread holds: rows up to 8192 wide
constexpr int kNormMaxWidth = kNormThreads * 4 * kNormVec;
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_kernel(const float* __restrict__ x, int32_t rows, int32_t hidden, const float* __restrict__ w,
                   float eps, uint32_t* __restrict__ out_bf16, float* __restrict__ out_f32,
                   const SeqEntry* __restrict__ seqs, uint32_t* __restrict__ out_split = nullptr) {
  SLMKV_TL(kTlNorm);
  const int row = blockIdx.x, tid = threadIdx.x;
  // The scale vector is a weight (no kernel writes it): fetched while the
  // previous kernel finishes, before the next kernel's weight copies queue
  // up in front of it.
  const int n4w = hidden / 4;
  const float4* wr = reinterpret_cast<const float4*>(w);
  float4 g4[kNormVec];
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    const int i = tid + j * kNormThreads;
    g4[j] = i < n4w ? wr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  wait_previous_kernel();
  if (row >= rows) return;
  const int src_row = seqs ? seqs[row].row_offset + seqs[row].count - 1 : row;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(src_row) * hidden);
  const int n4 = hidden / 4;
  float4 v[kNormVec];
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    const int i = tid + j * kNormThreads;
    v[j] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    s = fmaf(v[j].x, v[j].x, s);
    s = fmaf(v[j].y, v[j].y, s);
    s = fmaf(v[j].z, v[j].z, s);
    s = fmaf(v[j].w, v[j].w, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float part[kNormThreads / 32];
  if ((tid & 31) == 0) part[tid >> 5] = s;
  __syncthreads();
  s = 0.f;
#pragma unroll
  for (int k = 0; k < kNormThreads / 32; ++k) s += part[k];
  const float inv = 1.f / sqrtf(__fdiv_rn(s, static_cast<float>(hidden)) + eps);
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    const int i = tid + j * kNormThreads;
    if (i >= n4) break;
    const float4 g = g4[j];
    const float a = __fmul_rn(__fmul_rn(v[j].x, inv), g.x), b = __fmul_rn(__fmul_rn(v[j].y, inv), g.y);
    const float c = __fmul_rn(__fmul_rn(v[j].z, inv), g.z), d = __fmul_rn(__fmul_rn(v[j].w, inv), g.w);
    if (out_bf16)
      reinterpret_cast<uint2*>(out_bf16 + static_cast<size_t>(row) * (hidden / 2))[i] =
          make_uint2(pack_bf16x2(a, b), pack_bf16x2(c, d));
    else
      reinterpret_cast<float4*>(out_f32 + static_cast<size_t>(row) * hidden)[i] = make_float4(a, b, c, d);
    if (out_split) {
      // the row split hi = bf16(v), lo = bf16(v - hi), laid out for the
      // head GEMM's K order: 64-feature chunk c as [hi_c | lo_c] in the
      // first 2H, then hi again
      const uint2 hi = make_uint2(pack_bf16x2(a, b), pack_bf16x2(c, d));
      const float ha = __uint_as_float(hi.x << 16), hb = __uint_as_float(hi.x & 0xffff0000u);
      const float hc = __uint_as_float(hi.y << 16), hd = __uint_as_float(hi.y & 0xffff0000u);
      const uint2 lo = make_uint2(pack_bf16x2(__fsub_rn(a, ha), __fsub_rn(b, hb)),
                                  pack_bf16x2(__fsub_rn(c, hc), __fsub_rn(d, hd)));
      uint2* o = reinterpret_cast<uint2*>(out_split + static_cast<size_t>(row) * (3 * hidden / 2));
      o[32 * (i >> 4) + (i & 15)] = hi;
      o[32 * (i >> 4) + 16 + (i & 15)] = lo;
      o[2 * n4 + i] = hi;
    }
  }
}

// The split-bf16 vocabulary projection's weights: out [2H][V] bf16 =
// [hi; lo] of emb^T (emb [V][H] fp32), hi = bf16(w), lo = bf16(w - hi)
__global__ void head_split_kernel(const float* __restrict__ emb, int32_t V, int32_t H,
                                  __nv_bfloat16* __restrict__ out) {
  __shared__ float t[32][33];
  const int v0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int v = v0 + i, k = k0 + threadIdx.x;
    t[i][threadIdx.x] = (v < V && k < H) ? emb[static_cast<size_t>(v) * H + k] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int k = k0 + i, v = v0 + threadIdx.x;
    if (k >= H || v >= V) continue;
    const float w = t[threadIdx.x][i];
    const __nv_bfloat16 hi = __float2bfloat16_rn(w);
    const __nv_bfloat16 lo = __float2bfloat16_rn(__fsub_rn(w, __bfloat162float(hi)));
    out[static_cast<size_t>(k) * V + v] = hi;
    out[static_cast<size_t>(H + k) * V + v] = lo;
  }
}

// fp32 rows -> bf16 rows (round to nearest even), 4 values a thread.
__global__ void round_bf16_kernel(const float4* __restrict__ in, size_t n4, uint2* __restrict__ out) {
  SLMKV_TL(kTlRound);
  wait_previous_kernel();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float4 v = in[i];
    out[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

// situ_glu.rs:131-138
__device__ __forceinline__ float situ_sigmoid(float v) {
  if (v >= 0.f) return __fdiv_rn(1.f, __fadd_rn(1.f, libm::slm_expf(-v)));
  const float e = libm::slm_expf(v);
  return __fdiv_rn(e, __fadd_rn(1.f, e));
}
// situ_glu.rs:59-70 and :101-107: h = gate_act(gate) * up_act(up), as bf16
// (the down projection's rounded operand). gu rows are [gate | up].
__global__ void situ_kernel(const float* __restrict__ gu, int32_t rows, int32_t inter, float beta_gate,
                            float beta_up, uint32_t* __restrict__ h) {
  SLMKV_TL(kTlSitu);
  const size_t pairs = static_cast<size_t>(rows) * (inter / 2);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < pairs;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / (inter / 2), c = 2 * (i % (inter / 2));
    const float* row = gu + r * 2 * inter;
    float out[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float g = row[c + k], u = row[inter + c + k];
      const float ga = __fmul_rn(__fmul_rn(beta_gate, libm::slm_tanhf(__fdiv_rn(g, beta_gate))), situ_sigmoid(g));
      const float ua = __fmul_rn(beta_up, libm::slm_tanhf(__fdiv_rn(u, beta_up)));
      out[k] = __fmul_rn(ga, ua);
    }
    h[r * (inter / 2) + c / 2] = pack_bf16x2(out[0], out[1]);
  }
}

// ---- fused projections for up to kFusedRows token rows ------------------------
// Each output is the reference's own fold: sum = fma(x_k, w_k, sum) from 0
// over k in order (linear.rs:98-103), on bf16-rounded operands. A CTA stages
// kProjRows input rows, already in their rounded form, in shared memory;
// its 64 threads own 128 adjacent output columns (two each) and fold them for
// all staged rows (2 x kProjRows independent chains). The weights ([in][out]
// bf16 rows) stream through shared memory in 64-row chunks by cp.async, 128
// KiB in flight a CTA, so the folds never wait on one global load at a time.
//   kProjQKV   RMSNorm (attention_norm) fused in; writes q, k, v
//   kProjO     the attention output rounded here; adds onto the residual
//   kProjGU    RMSNorm (ffn_norm) fused in; gate and up columns j and I + j,
//              SiTU-GLU applied, h written as bf16 (the down projection's operand)
//   kProjDown  h as staged; adds onto the residual
// The RMSNorm square sum is the reference's sequential fma fold as well (one
// thread per staged row), so for f32 inputs the staged operands, and with
// them the projections, reproduce the reference bit for bit.
enum : int { kProjQKV = 0, kProjO = 1, kProjGU = 2, kProjDown = 3 };
constexpr int kProjThreads = 64;   // two output columns each
constexpr int kProjCols = 2 * kProjThreads;
constexpr int kProjRows = 4;       // token rows a CTA
constexpr int kProjChunk = 64;     // weight rows a stage
constexpr int kFusedRows = 1024;   // above this, tensor-core GEMMs
constexpr int kRowGemmRows = 512;  // up to this, this library's row GEMMs; beyond, cuBLAS

struct ProjArgs {
  const float* x;               // QKV, GU: residual stream; O: attention output  [rows, K] fp32
  const __nv_bfloat16* xh;      // Down: h  [rows, K] bf16
  const float* norm_w;          // QKV, GU: RMSNorm scale [K]
  float eps;
  int32_t rows, K;
  int32_t ncols;                // output columns this launch computes (QKV: H + 2KV; O, Down: H; GU: I)
  const __nv_bfloat16* w;       // [K][ld] bf16
  int32_t ld;
  float* y0;                    // QKV: q; O, Down: residual (accumulated)
  float* y1;                    // QKV: k
  float* y2;                    // QKV: v
  __nv_bfloat16* h;             // GU: [rows, I]
  int32_t H, KV, I;
  float beta_gate, beta_up;
  int32_t cols;                 // one-row kernel: output columns a CTA (a multiple of 8)
};

template <int MODE>
constexpr int proj_mats() {
  return MODE == kProjGU ? 2 : 1;  // gate and up slices
}
// weight chunks in flight: 128 KiB of weights a CTA either way
template <int MODE>
constexpr int proj_stages() {
  return proj_mats<MODE>() == 2 ? 4 : 8;
}
template <int MODE>
size_t proj_smem(int32_t K) {  // enough for either row blocking
  return static_cast<size_t>(kProjRows) * K * sizeof(float) +
         static_cast<size_t>(proj_stages<MODE>()) * proj_mats<MODE>() * kProjChunk * kProjCols * 2;
}

__device__ __forceinline__ float situ_gate(float g, float beta_gate) {
  return __fmul_rn(__fmul_rn(beta_gate, libm::slm_tanhf(__fdiv_rn(g, beta_gate))), situ_sigmoid(g));
}
__device__ __forceinline__ float situ_up(float u, float beta_up) {
  return __fmul_rn(beta_up, libm::slm_tanhf(__fdiv_rn(u, beta_up)));
}
__device__ __forceinline__ float round_bf16(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// NR: token rows a CTA (1 for a single-row step, else kProjRows; the last
// CTA may hold fewer).
template <int MODE, int NR>
__global__ void __launch_bounds__(kProjThreads) proj_kernel(const ProjArgs a) {
  SLMKV_TL(kTlProj);
  constexpr int NM = proj_mats<MODE>();
  constexpr int S = proj_stages<MODE>();
  extern __shared__ __align__(16) uint8_t smem[];
  float* xs = reinterpret_cast<float*>(smem);  // [kProjRows][K]
  const int K = a.K;
  __nv_bfloat16* wbuf = reinterpret_cast<__nv_bfloat16*>(smem + static_cast<size_t>(kProjRows) * K * 4);
  __shared__ float inv_s[NR];
  const int tid = threadIdx.x;
  const int r0 = blockIdx.y * NR;
  const int nr = min(NR, a.rows - r0);
  const int c0 = blockIdx.x * kProjCols;  // first output column of the CTA
  const int nchunks = (K + kProjChunk - 1) / kProjChunk;
  // weight rows [k0, k0 + kProjChunk) x columns [c0, c0 + 128) (and the up
  // columns I + c0 ...) into stage st, 16-byte copies; columns past ncols skip
  static_assert(kProjCols / 8 == 16, "16 segments of 8 columns a weight row");
  auto load_chunk = [&](int ch, int st) {
    const int k0 = ch * kProjChunk, nk = min(kProjChunk, K - k0);
#pragma unroll
    for (int m = 0; m < NM; ++m) {
      for (int i = tid; i < nk * 16; i += kProjThreads) {
        const int kr = i >> 4, seg = i & 15;
        const int col = c0 + 8 * seg;
        if (col < a.ncols)
          cp_async16(static_cast<uint32_t>(__cvta_generic_to_shared(
                         wbuf + ((st * NM + m) * kProjChunk + kr) * kProjCols + 8 * seg)),
                     a.w + static_cast<size_t>(k0 + kr) * a.ld + (m ? a.I : 0) + col);
      }
    }
    cp_async_commit();
  };
  for (int ch = 0; ch < S && ch < nchunks; ++ch) load_chunk(ch, ch);
  wait_previous_kernel();  // the rows come from the previous kernels
  // the rows as they arrive (coalesced), then, for the normed modes, the
  // reference's in-order square-sum fold over shared memory by one thread a
  // row (rmsnorm.rs:80-91) and the scaling and bf16 rounding in place
  for (int r = 0; r < nr; ++r) {
    const size_t row = static_cast<size_t>(r0 + r) * K;
    for (int k = tid; k < K; k += kProjThreads)
      xs[r * K + k] = MODE == kProjDown ? __bfloat162float(a.xh[row + k]) : a.x[row + k];
  }
  if (MODE == kProjQKV || MODE == kProjGU) {
    __syncthreads();
    if (tid < nr) {
      const float* xr = xs + tid * K;
      float s = 0.f;
#pragma unroll 8
      for (int k = 0; k < K; ++k) s = fmaf(xr[k], xr[k], s);
      inv_s[tid] = 1.f / sqrtf(__fdiv_rn(s, static_cast<float>(K)) + a.eps);
    }
    __syncthreads();
    for (int r = 0; r < nr; ++r)
      for (int k = tid; k < K; k += kProjThreads)
        xs[r * K + k] = round_bf16(__fmul_rn(__fmul_rn(xs[r * K + k], inv_s[r]), a.norm_w[k]));
  } else if (MODE == kProjO) {
    for (int r = 0; r < nr; ++r)
      for (int k = tid; k < K; k += kProjThreads) xs[r * K + k] = round_bf16(xs[r * K + k]);
  }
  const int c = c0 + 2 * tid;  // this thread's two columns
  float acc[NR][2], acc_up[NR][2];
#pragma unroll
  for (int r = 0; r < NR; ++r) acc[r][0] = acc[r][1] = acc_up[r][0] = acc_up[r][1] = 0.f;
  for (int ch = 0; ch < nchunks; ++ch) {
    const int st = ch % S;
    // chunk ch is complete once at most the S-1 groups issued after it are
    // pending; near the end fewer follow, so wait for all
    if (ch + S - 1 <= nchunks - 1) cp_async_wait<S - 1>();
    else cp_async_wait<0>();
    __syncthreads();  // chunk ch (and, the first time, the staged rows) visible
    const int k0 = ch * kProjChunk, nk = min(kProjChunk, K - k0);
    const uint32_t* wg = reinterpret_cast<const uint32_t*>(
        wbuf + (static_cast<size_t>(st) * NM) * kProjChunk * kProjCols) + tid;  // bf16 pairs
    const uint32_t* wu = wg + (NM > 1 ? kProjChunk * kProjCols / 2 : 0);
    if (c < a.ncols) {
      // groups of 8 k: every load of the group first, then the FMAs in k
      // order (nk is a multiple of 8: K and the chunk are)
      for (int kb = 0; kb < nk; kb += 8) {
        uint32_t wv[8], wuv[8];
        float xv[NR][8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          wv[j] = wg[(kb + j) * (kProjCols / 2)];
          if (MODE == kProjGU) wuv[j] = wu[(kb + j) * (kProjCols / 2)];
        }
#pragma unroll
        for (int r = 0; r < NR; ++r) {
          if (NR == 1 || r < nr) {
            const float4* xp = reinterpret_cast<const float4*>(xs + r * K + k0 + kb);
            const float4 lo = xp[0], hi = xp[1];
            xv[r][0] = lo.x, xv[r][1] = lo.y, xv[r][2] = lo.z, xv[r][3] = lo.w;
            xv[r][4] = hi.x, xv[r][5] = hi.y, xv[r][6] = hi.z, xv[r][7] = hi.w;
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float w0 = __uint_as_float(wv[j] << 16), w1 = __uint_as_float(wv[j] & 0xffff0000u);
          float u0 = 0.f, u1 = 0.f;
          if (MODE == kProjGU) {
            u0 = __uint_as_float(wuv[j] << 16);
            u1 = __uint_as_float(wuv[j] & 0xffff0000u);
          }
#pragma unroll
          for (int r = 0; r < NR; ++r) {
            if (NR == 1 || r < nr) {
              acc[r][0] = fmaf(xv[r][j], w0, acc[r][0]);
              acc[r][1] = fmaf(xv[r][j], w1, acc[r][1]);
              if (MODE == kProjGU) {
                acc_up[r][0] = fmaf(xv[r][j], u0, acc_up[r][0]);
                acc_up[r][1] = fmaf(xv[r][j], u1, acc_up[r][1]);
              }
            }
          }
        }
      }
    }
    __syncthreads();  // stage st is read: chunk ch + S may overwrite it
    if (ch + S < nchunks) load_chunk(ch + S, st);
  }
  if (c >= a.ncols) return;
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    if (r >= nr) break;
    const size_t row = static_cast<size_t>(r0 + r);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int col = c + e;
      if (MODE == kProjQKV) {
        if (col < a.H) a.y0[row * a.H + col] = acc[r][e];
        else if (col < a.H + a.KV) a.y1[row * a.KV + col - a.H] = acc[r][e];
        else a.y2[row * a.KV + col - a.H - a.KV] = acc[r][e];
      } else if (MODE == kProjGU) {
        // situ_glu.rs:101-107
        const float hv = __fmul_rn(situ_gate(acc[r][e], a.beta_gate), situ_up(acc_up[r][e], a.beta_up));
        a.h[row * a.I + col] = __float2bfloat16_rn(hv);
      } else {
        // transformer.rs add_residual_in_place: hidden += update
        float* y = a.y0 + row * a.ncols + col;
        *y = __fadd_rn(*y, acc[r][e]);
      }
    }
  }
}

// Many-row projections in the reference's order (the exact-order path at 2 ..
// 1024 rows): one CTA of 128 threads computes a tile of BM = 8 TM rows x 64
// output columns, each thread TM rows x 4 columns, every output the same
// in-order fma fold over k from 0, over the same bf16-rounded operands, as
// proj_kernel's (linear.rs:98-103): the results are proj_kernel's bit for
// bit. The CTA's rows sit transposed in shared memory for the whole K
// ([k][row]; for the normed modes the square sums folded in order by one
// thread a row, then scaled and rounded in place); the weights stream
// through a ring of 32-row chunks (cp.async), the first ones requested before
// waiting on the previous kernel. A k step is one shared load of the TM row
// values, one of the 4 weights, 4 TM fmas; proj_kernel's 64-thread CTAs of 4
// rows re-read every weight for every 4 rows at 2 warps an SM. GU: a tile is
// 32 gate and the 32 matching up columns; a thread holds 2 of each and
// applies SiTU-GLU. K must be a multiple of 32.
constexpr int kPtThreads = 128;
constexpr int kPtCols = 64;   // output columns a tile (GU: 32 gate + 32 up)
constexpr int kPtChunk = 32;  // weight rows a ring stage
constexpr int kPtStages = 4;
__host__ __device__ constexpr int pt_rows(int tm) { return 8 * tm; }
__host__ __device__ constexpr int pt_ld(int tm) { return 8 * tm + 4; }  // padded length of a [k] row
// FULL: the CTA's whole weight slice (K x 64 columns) is requested before
// the wait and stays in shared memory (for grids of few CTAs, where the
// ring's refills would sit on the fold's path); else the 4-stage ring
template <int TM>
size_t projt_smem(int32_t K, bool full = false) {
  return static_cast<size_t>(K) * pt_ld(TM) * 4 +
         static_cast<size_t>(full ? K / kPtChunk : kPtStages) * kPtChunk * kPtCols * 2;
}

template <int MODE, int TM, bool FULL>
__global__ void __launch_bounds__(kPtThreads) projt_kernel(const ProjArgs a) {
  SLMKV_TL(kTlProj);
  constexpr int BM = pt_rows(TM), LDA = pt_ld(TM);
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = a.K, tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  float* xs = reinterpret_cast<float*>(smem);  // [K][LDA]
  uint16_t* wb = reinterpret_cast<uint16_t*>(smem + static_cast<size_t>(K) * LDA * 4);  // [stage][32][64]
  __shared__ float inv_s[BM];
  const int r0 = blockIdx.y * BM, nr = min(BM, a.rows - r0);
  const int nchunks = K / kPtChunk;
  // the tile's weight columns: QKV, O, Down 64 adjacent; GU 32 gate columns
  // c0 .. and the up columns I + c0 ..
  const int c0 = MODE == kProjGU ? blockIdx.x * (kPtCols / 2) : blockIdx.x * kPtCols;
  auto load_chunk = [&](int ch, int st) {
    // 32 weight rows x 8 segments of 8 columns: two 16-byte copies a thread
    for (int i = tid; i < kPtChunk * 8; i += kPtThreads) {
      const int kr = i >> 3, seg = i & 7;
      const int lc = MODE == kProjGU ? c0 + 8 * (seg & 3) : c0 + 8 * seg;  // output column
      const int col = MODE == kProjGU && seg >= 4 ? a.I + lc : lc;          // weight column
      if (lc < a.ncols)
        cp_async16(static_cast<uint32_t>(__cvta_generic_to_shared(wb + (st * kPtChunk + kr) * kPtCols + 8 * seg)),
                   a.w + static_cast<size_t>(ch * kPtChunk + kr) * a.ld + col);
    }
    cp_async_commit();
  };
  if constexpr (FULL) {
    for (int ch = 0; ch < nchunks; ++ch) load_chunk(ch, ch);  // one group a chunk
  } else {
    for (int ch = 0; ch < kPtStages - 1; ++ch) {
      if (ch < nchunks) load_chunk(ch, ch);
      else cp_async_commit();
    }
  }
  wait_previous_kernel();  // the rows come from the previous kernels
  // the rows, transposed: a thread takes features k, k + 128, ... and for
  // each all BM rows (coalesced across the threads), KI features' loads in
  // flight before their stores; rows past the end are zeros
  constexpr int KI = TM == 4 ? 2 : 4;
  for (int kb = 0; kb < K; kb += KI * kPtThreads) {
    float v[KI][BM];
#pragma unroll
    for (int u = 0; u < KI; ++u) {
      const int k = kb + u * kPtThreads + tid;
#pragma unroll
      for (int r = 0; r < BM; ++r) {
        v[u][r] = 0.f;
        if (k < K && r < nr) {
          const size_t src = static_cast<size_t>(r0 + r) * K + k;
          v[u][r] = MODE == kProjDown ? __bfloat162float(a.xh[src]) : a.x[src];
        }
      }
    }
#pragma unroll
    for (int u = 0; u < KI; ++u) {
      const int k = kb + u * kPtThreads + tid;
      if (k < K) {
#pragma unroll
        for (int r = 0; r < BM; r += 4)
          *reinterpret_cast<float4*>(xs + k * LDA + r) = make_float4(v[u][r], v[u][r + 1], v[u][r + 2], v[u][r + 3]);
      }
    }
  }
  __syncthreads();
  if (MODE == kProjQKV || MODE == kProjGU) {
    if (tid < nr) {  // rmsnorm.rs:80-91: the square sum in order
      float s = 0.f;
#pragma unroll 8
      for (int k = 0; k < K; ++k) s = fmaf(xs[k * LDA + tid], xs[k * LDA + tid], s);
      inv_s[tid] = 1.f / sqrtf(__fdiv_rn(s, static_cast<float>(K)) + a.eps);
    }
    __syncthreads();
    for (int k = tid; k < K; k += kPtThreads) {
      const float g = a.norm_w[k];
      for (int r = 0; r < nr; ++r) xs[k * LDA + r] = round_bf16(__fmul_rn(__fmul_rn(xs[k * LDA + r], inv_s[r]), g));
    }
  } else if (MODE == kProjO) {
    for (int k = tid; k < K; k += kPtThreads)
      for (int r = 0; r < nr; ++r) xs[k * LDA + r] = round_bf16(xs[k * LDA + r]);
  }
  float acc[TM][4];
#pragma unroll
  for (int i = 0; i < TM; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  if constexpr (FULL) {
    cp_async_wait<0>();
    __syncthreads();
  }
  for (int ch = 0; ch < nchunks; ++ch) {
    const int st = FULL ? ch : ch % kPtStages;
    if constexpr (!FULL) {
      // the stage chunk ch + 3 fills was read in the previous iteration,
      // which ended with a barrier
      if (ch + kPtStages - 1 < nchunks) load_chunk(ch + kPtStages - 1, (ch + kPtStages - 1) % kPtStages);
      else cp_async_commit();
      cp_async_wait<kPtStages - 1>();  // chunk ch landed (this thread's copies)
      __syncthreads();                 // ... and every thread's; the rows, the first time
    }
    const uint16_t* wst = wb + st * kPtChunk * kPtCols;
    const float* xk = xs + static_cast<size_t>(ch) * kPtChunk * LDA + ty * TM;
#pragma unroll 8
    for (int kk = 0; kk < kPtChunk; ++kk) {
      float xv[TM];
      if constexpr (TM == 4) {
        const float4 v = *reinterpret_cast<const float4*>(xk + kk * LDA);
        xv[0] = v.x, xv[1] = v.y, xv[2] = v.z, xv[3] = v.w;
      } else {
        xv[0] = xk[kk * LDA];
      }
      uint32_t w01, w23;
      if (MODE == kProjGU) {  // a gate pair, the matching up pair
        w01 = *reinterpret_cast<const uint32_t*>(wst + kk * kPtCols + 2 * tx);
        w23 = *reinterpret_cast<const uint32_t*>(wst + kk * kPtCols + 32 + 2 * tx);
      } else {
        const uint2 w = *reinterpret_cast<const uint2*>(wst + kk * kPtCols + 4 * tx);
        w01 = w.x, w23 = w.y;
      }
      const float w0 = __uint_as_float(w01 << 16), w1 = __uint_as_float(w01 & 0xffff0000u);
      const float w2 = __uint_as_float(w23 << 16), w3 = __uint_as_float(w23 & 0xffff0000u);
#pragma unroll
      for (int i = 0; i < TM; ++i) {
        acc[i][0] = fmaf(xv[i], w0, acc[i][0]);
        acc[i][1] = fmaf(xv[i], w1, acc[i][1]);
        acc[i][2] = fmaf(xv[i], w2, acc[i][2]);
        acc[i][3] = fmaf(xv[i], w3, acc[i][3]);
      }
    }
    if constexpr (!FULL) __syncthreads();  // stage st is read: a later chunk may overwrite it
  }
  cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int r = ty * TM + i;
    if (r >= nr) break;
    const size_t row = static_cast<size_t>(r0 + r);
    if (MODE == kProjGU) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = c0 + 2 * tx + e;
        if (col < a.ncols)  // situ_glu.rs:101-107
          a.h[row * a.I + col] = __float2bfloat16_rn(
              __fmul_rn(situ_gate(acc[i][e], a.beta_gate), situ_up(acc[i][2 + e], a.beta_up)));
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = c0 + 4 * tx + e;
        if (col >= a.ncols) continue;
        if (MODE == kProjQKV) {
          if (col < a.H) a.y0[row * a.H + col] = acc[i][e];
          else if (col < a.H + a.KV) a.y1[row * a.KV + col - a.H] = acc[i][e];
          else a.y2[row * a.KV + col - a.H - a.KV] = acc[i][e];
        } else {  // transformer.rs add_residual_in_place: hidden += update
          float* y = a.y0 + row * a.ncols + col;
          *y = __fadd_rn(*y, acc[i][e]);
        }
      }
    }
  }
}

// Shared memory above 48 KB is opted into per device and kernel, raised to
// the largest launch so far.
template <int MODE, int TM, bool FULL>
cudaError_t launch_projt(const ProjArgs& a, cudaStream_t s) {
  static size_t configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64) return cudaErrorInvalidDevice;
  const size_t smem = projt_smem<TM>(a.K, FULL);
  if (smem > configured[dev]) {
    e = cudaFuncSetAttribute(projt_kernel<MODE, TM, FULL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = smem;
  }
  const int cols = MODE == kProjGU ? kPtCols / 2 : kPtCols;
  return launch_chained(projt_kernel<MODE, TM, FULL>,
                        dim3((a.ncols + cols - 1) / cols, (a.rows + pt_rows(TM) - 1) / pt_rows(TM)),
                        dim3(kPtThreads), smem, s, a);
}
// the whole slice when the grid's CTAs all fit at once with it (one wave)
template <int MODE, int TM>
cudaError_t launch_projt_best(const ProjArgs& a, cudaStream_t s, int64_t ctas) {
  const size_t full = projt_smem<TM>(a.K, true);
  const int64_t per_sm = full <= 227 * 1024 ? (228 * 1024) / static_cast<int64_t>(full + 1024) : 0;
  if (per_sm > 0 && ctas <= 148 * per_sm) return launch_projt<MODE, TM, true>(a, s);
  return launch_projt<MODE, TM, false>(a, s);
}

// linear.rs:119-152, the tied vocabulary projection (fp32, unrounded), for
// up to 64 rows: logits[r][v] = sum_k x[r][k] emb[v][k]. A CTA stages 8 rows
// in shared memory (small enough for two CTAs an SM, so that enough
// embedding loads are in flight); a warp takes 4 vocabulary entries at a
// time, its lanes 4 features apart (coalesced 16-byte loads of the embedding
// rows, the next step's issued before this step's FMAs), 32 sums a lane,
// then a reduce-scatter across the lanes (5 exchange
// steps, each halving the sums a lane holds: lane l ends with row l / 4,
// entry l % 4). CTAs of the other row groups read the same embedding rows at
// the same time (from L2).
constexpr int kHeadThreads = 256;
constexpr int kHeadRows = 8;       // rows a CTA
constexpr int kHeadEntries = 64;   // vocabulary entries a CTA: 8 warps x 4, two rounds
constexpr int kHeadMaxRows = 64;
constexpr int kHeadMaxWidth = 4096;  // 8 rows x 16 KiB of shared memory
template <int N>
__device__ __forceinline__ void head_halve(float (&a)[32], int lane, int o) {
  const bool upper = (lane & o) != 0;
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    const float send = upper ? a[i] : a[i + N / 2];
    const float keep = upper ? a[i + N / 2] : a[i];
    a[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
  }
}
__global__ void __launch_bounds__(kHeadThreads, 2) head_kernel(const float* __restrict__ x, int32_t rows, int32_t H,
                                                            const float* __restrict__ emb, int32_t V,
                                                            float* __restrict__ logits) {
  SLMKV_TL(kTlHead);
  wait_previous_kernel();
  extern __shared__ float4 head_x[];  // [kHeadRows][H / 4]
  const int n4 = H / 4;
  const int r0 = blockIdx.y * kHeadRows, nr = min(kHeadRows, rows - r0);
  const float4* x4 = reinterpret_cast<const float4*>(x);
  for (int r = 0; r < kHeadRows; ++r)
    for (int k = threadIdx.x; k < n4; k += kHeadThreads)
      head_x[r * n4 + k] = r < nr ? x4[static_cast<size_t>(r0 + r) * n4 + k] : make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float4* e4 = reinterpret_cast<const float4*>(emb);
#pragma unroll 1
  for (int round = 0; round < kHeadEntries / 32; ++round) {
    const int v0 = blockIdx.x * kHeadEntries + round * 32 + warp * 4;
    if (v0 >= V) break;  // warp-uniform
    float a[32];  // a[4 r + j]: row r, entry v0 + j
#pragma unroll
    for (int i = 0; i < 32; ++i) a[i] = 0.f;
    const float4* ev[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) ev[j] = e4 + static_cast<size_t>(min(v0 + j, V - 1)) * n4;
    // the next step's embedding loads are issued before this step's FMAs
    float4 e[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) e[j] = lane < n4 ? __ldcg(ev[j] + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = lane; k < n4; k += 32) {
      float4 en[4];
      const bool more = k + 32 < n4;
#pragma unroll
      for (int j = 0; j < 4; ++j) en[j] = more ? __ldcg(ev[j] + k + 32) : e[j];
#pragma unroll
      for (int r = 0; r < kHeadRows; ++r) {
        const float4 xv = head_x[r * n4 + k];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float t = a[4 * r + j];
          t = fmaf(xv.x, e[j].x, t);
          t = fmaf(xv.y, e[j].y, t);
          t = fmaf(xv.z, e[j].z, t);
          a[4 * r + j] = fmaf(xv.w, e[j].w, t);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) e[j] = en[j];
    }
    head_halve<32>(a, lane, 16);
    head_halve<16>(a, lane, 8);
    head_halve<8>(a, lane, 4);
    head_halve<4>(a, lane, 2);
    head_halve<2>(a, lane, 1);
    const int r = lane >> 2, j = lane & 3;  // a[0] is sum `lane`
    if (r < nr && v0 + j < V) logits[static_cast<size_t>(r0 + r) * V + v0 + j] = a[0];
  }
}

// greedy.rs argmax_finite, one CTA per row: the first maximal logit; a
// non-finite logit sets the context's error bit (the step then fails).
constexpr int kArgmaxThreads = 256;
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float* __restrict__ logits,
                                                                int32_t vocab, int32_t* __restrict__ next,
                                                                int32_t* __restrict__ err) {
  SLMKV_TL(kTlArgmax);
  wait_previous_kernel();
  const float* row = logits + static_cast<size_t>(blockIdx.x) * vocab;
  float best = -INFINITY;
  int32_t idx = 0x7fffffff;
  bool bad = false;
  for (int i = threadIdx.x; i < vocab; i += kArgmaxThreads) {
    const float v = row[i];
    if (!isfinite(v)) bad = true;
    if (idx == 0x7fffffff || v > best) {  // strictly greater: the earlier index stays
      best = v;
      idx = i;
    }
  }
  // (value, index) pairs: larger value wins, then the smaller index
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) {
      best = ob;
      idx = oi;
    }
  }
  __shared__ float sb[kArgmaxThreads / 32];
  __shared__ int32_t si[kArgmaxThreads / 32];
  const bool any_bad = __syncthreads_or(bad);
  if ((threadIdx.x & 31) == 0) {
    sb[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < kArgmaxThreads / 32; ++k)
      if (sb[k] > best || (sb[k] == best && si[k] < idx)) {
        best = sb[k];
        idx = si[k];
      }
    if (any_bad) {
      atomicOr(err, kErrLogits);
      idx = 0;
    }
    next[blockIdx.x] = idx;
  }
}

}  // namespace
}  // namespace slmkv

struct slm_model {
  slm_ctx* ctx = nullptr;
  int32_t V = 0, H = 0, I = 0, L = 0, KV = 0;
  float eps = 0.f, beta_gate = 0.f, beta_up = 0.f;
  // steps of up to this many token rows run the fused exact-order
  // projections; 0 when their shared memory does not fit this model
  int32_t exact_rows = 0;
  bool exact_fits = false;
  // f32 pool: the exact-order steps also attend in the reference's order
  // (slm_batch_attention_exact), so that their logits are the CPU path's
  bool f32_pool = false;
  bool head_kernel_ok = false;  // rows up to 64 on head_kernel (hidden <= 4096)
  // one-row steps: columns a CTA of proj1_kernel per mode (0: proj_kernel)
  int32_t p1_cols[4] = {0, 0, 0, 0};
  bool mlp1_ok = false;  // one-row steps: output .. down projection as one cluster launch
  bool mlp1_qkv_ok = false;  // ... and the next layer's norm and q/k/v too
  cublasHandle_t blas = nullptr;
  void* weights = nullptr;  // one device allocation for every tensor
  const float* emb = nullptr;         // [V, H] fp32: lookup table and tied vocabulary projection
  const float* final_norm = nullptr;  // [H]
  // Projection matrices bf16 and transposed ([in][out] rows): wqkv [H][H+2KV]
  // (columns q | k | v), wo [H][H], wgu [H][2I] (columns gate | up), wd [I][H].
  // the tied head for the row-GEMM path (models of hidden >= 512): [2H][V]
  // bf16 (hi; lo of emb^T) and its tensor map; null otherwise
  __nv_bfloat16* head3 = nullptr;
  CUtensorMap tm_head;
  struct Layer {
    const float *attn_norm, *ffn_norm;  // [H]
    const __nv_bfloat16 *wqkv, *wo, *wgu, *wd;
    CUtensorMap tm_qkv, tm_o, tm_gu, tm_d;  // the same matrices for the tensor-core row GEMMs
    // Models whose one-row steps run as one cluster launch a layer: the same
    // matrices bf16 in the reference's [out][in] layout (each output's
    // weights one contiguous row): wqkv_r [H+2KV][H], wo_r [H][H],
    // wgu_r [2I][H] (gate rows, then up), wd_r [H][I]; null otherwise.
    const __nv_bfloat16 *wqkv_r, *wo_r, *wgu_r, *wd_r;
  };
  std::vector<Layer> layers;
  int32_t sms = 148;
  // scratch, grown on demand: rows for token rows, out rows for projected rows
  int32_t rows_cap = 0, out_cap = 0;
  float *x = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *gu = nullptr;
  uint32_t* xb = nullptr;  // bf16 pairs, [rows, max(H, I) / 2]
  uint32_t* xs3 = nullptr;  // bf16 pairs, [out rows, 3H / 2]: the split head operand
  uint32_t* hb = nullptr;  // bf16 pairs, [rows, I / 2]: the row GEMMs' SiTU-GLU output
  // the row GEMMs' RMSNorm across the projections: bf16(x * g) [rows, H] and
  // each row's square sums over the 128-column tiles [rows, ceil(H / 128)]
  __nv_bfloat16* xg = nullptr;
  float* ssq = nullptr;

  float *xf = nullptr, *logits = nullptr;
};

namespace slmkv {
namespace {

// linear.rs:14-23 on the bits (non-finite values keep their leading bits).
uint16_t bf16_bits(float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  if ((b & 0x7f800000u) == 0x7f800000u) return static_cast<uint16_t>((b & 0x007fffffu) ? 0x7fc0u : (b >> 16));
  b += 0x7fffu + ((b >> 16) & 1u);
  return static_cast<uint16_t>(b >> 16);
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

slm_status cuda_fail(slm_ctx* c, const char* what, cudaError_t e) {
  std::string m = std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e);
  return ctx_fail(c, SLM_ERR_CUDA, m.c_str());
}
slm_status blas_fail(slm_ctx* c, const char* what, cublasStatus_t e) {
  std::string m = std::string("CUDA error in ") + what + ": cuBLAS status " + std::to_string(static_cast<int>(e));
  return ctx_fail(c, SLM_ERR_CUDA, m.c_str());
}

void free_scratch(slm_model* m) {
  for (void* p : {static_cast<void*>(m->x), static_cast<void*>(m->q), static_cast<void*>(m->k),
                  static_cast<void*>(m->v), static_cast<void*>(m->att), static_cast<void*>(m->gu),
                  static_cast<void*>(m->xb), static_cast<void*>(m->hb), static_cast<void*>(m->xf),
                  static_cast<void*>(m->logits), static_cast<void*>(m->xg), static_cast<void*>(m->ssq),
                  static_cast<void*>(m->xs3)})
    if (p) cudaFree(p);
  m->x = m->q = m->k = m->v = m->att = m->gu = m->xf = m->logits = m->ssq = nullptr;
  m->xb = m->hb = m->xs3 = nullptr;
  m->xg = nullptr;
  m->rows_cap = m->out_cap = 0;
}

// the row GEMMs' 128-column output tiles across the hidden width
int32_t ssq_tiles(int32_t H) { return (H + 127) / 128; }

// Scratch for `rows` token rows and `out_rows` projected rows (the stream
// is synchronized before buffers are replaced).
slm_status ensure_scratch(slm_model* m, int32_t rows, int32_t out_rows, cudaStream_t s) {
  if (rows <= m->rows_cap && out_rows <= m->out_cap) return SLM_OK;
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(m->ctx, "slm_model step", e);
  const int32_t r = std::max(rows, m->rows_cap), o = std::max(out_rows, m->out_cap);
  free_scratch(m);
  const size_t R = static_cast<size_t>(r), O = static_cast<size_t>(o);
  const size_t wide = static_cast<size_t>(std::max(m->H, m->I));
  struct A {
    void** p;
    size_t bytes;
  } allocs[] = {{reinterpret_cast<void**>(&m->x), R * m->H * 4},
                {reinterpret_cast<void**>(&m->q), R * m->H * 4},
                {reinterpret_cast<void**>(&m->k), R * m->KV * 4},
                {reinterpret_cast<void**>(&m->v), R * m->KV * 4},
                {reinterpret_cast<void**>(&m->att), R * m->H * 4},
                {reinterpret_cast<void**>(&m->gu), R * 2 * m->I * 4},
                {reinterpret_cast<void**>(&m->xb), R * wide * 2},
                {reinterpret_cast<void**>(&m->hb), R * m->I * 2},
                {reinterpret_cast<void**>(&m->xg), R * m->H * 2},
                {reinterpret_cast<void**>(&m->ssq), R * ssq_tiles(m->H) * 4},
                {reinterpret_cast<void**>(&m->xf), O * m->H * 4},
                {reinterpret_cast<void**>(&m->xs3), O * 3 * m->H * 2},
                {reinterpret_cast<void**>(&m->logits), O * m->V * 4}};
  for (const A& a : allocs) {
    e = cudaMalloc(a.p, a.bytes);
    if (e != cudaSuccess) {
      free_scratch(m);
      return cuda_fail(m->ctx, "slm_model scratch allocation", e);
    }
  }
  m->rows_cap = r;
  m->out_cap = o;
  return SLM_OK;
}

// y[rows, N] (+)= x[rows, K] . wT[K, col0 : col0 + N] (transposed bf16 weights
// with row length ld, passed at col0), bf16 operands, fp32 accumulation.
cublasStatus_t gemm_t(cublasHandle_t h, const void* x, int32_t rows, int32_t K, const __nv_bfloat16* wT,
                      int32_t ld, int32_t N, float* y, float beta) {
  const float alpha = 1.f;
  return cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_N, N, rows, K, &alpha, wT, CUDA_R_16BF, ld, x, CUDA_R_16BF,
                      K, &beta, y, CUDA_R_32F, N, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
}

int32_t grid_for(size_t work, int32_t threads) {
  const size_t g = (work + threads - 1) / threads;
  return static_cast<int32_t>(std::min<size_t>(std::max<size_t>(g, 1), 148 * 16));
}

// ---- one token row (batch-1 decode) ----------------------------------------------
// The fold of one output column is K dependent fmas in k order and cannot be
// split, so a one-row projection is a few hundred independent folds; the
// kernel above packs 128 columns (two a thread, four for gate/up) into each
// of 64 threads and issues them from a handful of CTAs, and each warp's
// long dependent instruction stream sets the time. Here every thread folds one
// column (gate/up: the first `cols` threads the gate columns, the next the
// up columns), a CTA takes `cols` columns, and the projection spreads over
// ncols / cols small CTAs. The CTA's whole weight tile (K rows x cols
// columns, bf16) is requested by cp.async before waiting on the previous
// kernel (weights are immutable), so it lands while that kernel finishes.
// Same operands, folds, norm and epilogues as proj_kernel: the same bits.
constexpr int kProj1MaxSmem = 200 * 1024;
template <int MODE>
size_t proj1_smem(int32_t K, int32_t cols) {
  return static_cast<size_t>(K) * 4 + static_cast<size_t>(proj_mats<MODE>()) * K * cols * 2;
}
// Columns a CTA: 32 (gate/up and down: more CTAs for the larger matrices) or
// 64, halved while the tile does not fit; 0 when not even 8 fit.
template <int MODE>
int32_t proj1_cols(int32_t K) {
  int32_t c = (MODE == kProjQKV || MODE == kProjO) ? 64 : 32;
  while (c >= 8 && proj1_smem<MODE>(K, c) > static_cast<size_t>(kProj1MaxSmem)) c /= 2;
  return c >= 8 ? c : 0;
}

template <int MODE>
__global__ void __launch_bounds__(128) proj1_kernel(const ProjArgs a) {
  SLMKV_TL(kTlProj1);
  constexpr int NM = proj_mats<MODE>();
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = a.K, C = a.cols, NT = NM * C;
  float* xs = reinterpret_cast<float*>(smem);  // [K]
  __nv_bfloat16* ws = reinterpret_cast<__nv_bfloat16*>(smem + static_cast<size_t>(K) * 4);  // [NM][K][C]
  __shared__ float inv_s;
  __shared__ float up_s[64];
  const int tid = threadIdx.x;
  const int c0 = blockIdx.x * C;
  const int seg = C / 8;  // 16-byte segments of a weight row
  for (int i = tid; i < NM * K * seg; i += NT) {
    const int m = i / (K * seg), rem = i - m * K * seg;
    const int k = rem / seg, sg = rem - k * seg;
    const int col = c0 + 8 * sg;
    if (col < a.ncols)
      cp_async16(static_cast<uint32_t>(__cvta_generic_to_shared(ws + (static_cast<size_t>(m) * K + k) * C + 8 * sg)),
                 a.w + static_cast<size_t>(k) * a.ld + (m ? a.I : 0) + col);
  }
  cp_async_commit();
  wait_previous_kernel();  // the row comes from the previous kernels
  for (int k = tid; k < K; k += NT) xs[k] = MODE == kProjDown ? __bfloat162float(a.xh[k]) : a.x[k];
  __syncthreads();
  if (MODE == kProjQKV || MODE == kProjGU) {
    if (tid == 0) {  // rmsnorm.rs:80-91, the in-order square-sum fold
      float sum = 0.f;
#pragma unroll 8
      for (int k = 0; k < K; ++k) sum = fmaf(xs[k], xs[k], sum);
      inv_s = 1.f / sqrtf(__fdiv_rn(sum, static_cast<float>(K)) + a.eps);
    }
    __syncthreads();
    for (int k = tid; k < K; k += NT) xs[k] = round_bf16(__fmul_rn(__fmul_rn(xs[k], inv_s), a.norm_w[k]));
  } else if (MODE == kProjO) {
    for (int k = tid; k < K; k += NT) xs[k] = round_bf16(xs[k]);
  }
  cp_async_wait<0>();
  __syncthreads();
  const int m = (NM > 1 && tid >= C) ? 1 : 0;
  const int cl = tid - m * C, col = c0 + cl;
  float acc = 0.f;
  if (col < a.ncols) {
    const uint16_t* wc = reinterpret_cast<const uint16_t*>(ws) + static_cast<size_t>(m) * K * C + cl;
    for (int k = 0; k < K; k += 8) {  // K is a multiple of 8; loads first, then the fmas in order
      const float4 x0 = *reinterpret_cast<const float4*>(xs + k);
      const float4 x1 = *reinterpret_cast<const float4*>(xs + k + 4);
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = wc[static_cast<size_t>(k + j) * C];
      acc = fmaf(x0.x, __uint_as_float(w[0] << 16), acc);
      acc = fmaf(x0.y, __uint_as_float(w[1] << 16), acc);
      acc = fmaf(x0.z, __uint_as_float(w[2] << 16), acc);
      acc = fmaf(x0.w, __uint_as_float(w[3] << 16), acc);
      acc = fmaf(x1.x, __uint_as_float(w[4] << 16), acc);
      acc = fmaf(x1.y, __uint_as_float(w[5] << 16), acc);
      acc = fmaf(x1.z, __uint_as_float(w[6] << 16), acc);
      acc = fmaf(x1.w, __uint_as_float(w[7] << 16), acc);
    }
  }
  if (MODE == kProjGU) {
    if (m == 1) up_s[cl] = acc;
    __syncthreads();
    if (m == 0 && col < a.ncols)  // situ_glu.rs:101-107
      a.h[col] = __float2bfloat16_rn(__fmul_rn(situ_gate(acc, a.beta_gate), situ_up(up_s[cl], a.beta_up)));
    return;
  }
  if (col >= a.ncols) return;
  if (MODE == kProjQKV) {
    if (col < a.H) a.y0[col] = acc;
    else if (col < a.H + a.KV) a.y1[col - a.H] = acc;
    else a.y2[col - a.H - a.KV] = acc;
  } else {  // transformer.rs add_residual_in_place: hidden += update
    a.y0[col] = __fadd_rn(a.y0[col], acc);
  }
}

// ---------------------------------------------------------------------------
// One-row steps: a layer's output projection, FFN RMSNorm, gate/up with
// SiTU-GLU and down projection in one launch of one thread-block cluster
// (transformer.rs:221-292 after the attention). Each of the kMlpCluster CTAs
// holds its slice of the three weight matrices in shared memory (requested
// before waiting on the attention kernel) and computes its slice of the
// output columns, each the reference's in-order fma fold (linear.rs:98-103)
// as proj1_kernel does; the new residual row and the SiTU-GLU outputs are
// written into every CTA's shared memory (distributed shared memory) and a
// cluster barrier stands where two kernel boundaries stood. The slices are
// the matrices' [out][in] copies, one padded row an output column, so a fold
// reads 8 weights with one 16-byte shared load.
constexpr int kMlpCluster = 8;
constexpr int kMlpThreads = 192;
struct MlpArgs {
  const float* att;          // attention output row [H]
  float* x;                  // residual row [H]: + output projection, + down projection
  const __nv_bfloat16* wo;   // [H out][H in]
  const __nv_bfloat16* wgu;  // [2I out][H in]: gate rows, then up rows
  const __nv_bfloat16* wd;   // [H out][I in]
  const float* ffn_norm;     // [H]
  float eps, beta_gate, beta_up;
  int32_t H, I;
  // with wqkv set: the next layer's attention RMSNorm and q/k/v projection too
  const __nv_bfloat16* wqkv;  // [H + 2 KV out][H in]
  const float* attn_norm;     // [H]
  float *q, *k, *v;           // [H], [KV], [KV]
  int32_t KV;
};
// Shared memory of one CTA (KV = 0: without the next q/k/v): the bf16 slices
// [CO][H + 8] output, [CI][H + 8] gate and up, [CO][I + 8] down, [CQ][H + 8]
// q/k/v, then the f32 rows (rounded attention row, residual, normalised row,
// SiTU-GLU outputs, this CTA's up columns, the FFN and attention norm scales)
size_t mlp1_smem(int32_t H, int32_t I, int32_t KV) {
  const size_t co = H / kMlpCluster, ci = I / kMlpCluster;
  const size_t cq = KV ? (H + 2 * KV) / kMlpCluster : 0;
  const size_t hp = static_cast<size_t>(H) + 8, ip = static_cast<size_t>(I) + 8;
  return 2 * (co * hp + 2 * ci * hp + co * ip + cq * hp) +
         4 * (4 * static_cast<size_t>(H) + I + ci + (KV ? H : 0));
}
bool mlp1_fits(int32_t H, int32_t I, int32_t KV) {
  return H % (8 * kMlpCluster) == 0 && I % (8 * kMlpCluster) == 0 && H % 8 == 0 &&
         2 * (I / kMlpCluster) <= kMlpThreads && H / kMlpCluster <= kMlpThreads &&
         (KV == 0 || ((H + 2 * KV) % (8 * kMlpCluster) == 0 &&
                      (H + 2 * KV) / kMlpCluster <= kMlpThreads)) &&
         mlp1_smem(H, I, KV) <= 227 * 1024;
}
// acc = fold over k of x[k] * w[k] (bf16 row w, 16-byte aligned), in order;
// K % 8 == 0
__device__ __forceinline__ float fold_row(const uint16_t* w, const float* x, int K) {
  float acc = 0.f;
#pragma unroll 4
  for (int k = 0; k < K; k += 8) {
    const uint4 wv = *reinterpret_cast<const uint4*>(w + k);
    const float4 x0 = *reinterpret_cast<const float4*>(x + k);
    const float4 x1 = *reinterpret_cast<const float4*>(x + k + 4);
    acc = fmaf(x0.x, __uint_as_float(wv.x << 16), acc);
    acc = fmaf(x0.y, __uint_as_float(wv.x & 0xffff0000u), acc);
    acc = fmaf(x0.z, __uint_as_float(wv.y << 16), acc);
    acc = fmaf(x0.w, __uint_as_float(wv.y & 0xffff0000u), acc);
    acc = fmaf(x1.x, __uint_as_float(wv.z << 16), acc);
    acc = fmaf(x1.y, __uint_as_float(wv.z & 0xffff0000u), acc);
    acc = fmaf(x1.z, __uint_as_float(wv.w << 16), acc);
    acc = fmaf(x1.w, __uint_as_float(wv.w & 0xffff0000u), acc);
  }
  return acc;
}
// rmsnorm.rs:80-91's in-order square-sum fold and 1 / sqrt(mean + eps)
__device__ __forceinline__ float inv_rms(const float* x, int H, float eps) {
  float sum = 0.f;
  const float4* x4 = reinterpret_cast<const float4*>(x);
#pragma unroll 4
  for (int k = 0; k < H / 4; ++k) {
    const float4 v = x4[k];
    sum = fmaf(v.x, v.x, sum);
    sum = fmaf(v.y, v.y, sum);
    sum = fmaf(v.z, v.z, sum);
    sum = fmaf(v.w, v.w, sum);
  }
  return 1.f / sqrtf(__fdiv_rn(sum, static_cast<float>(H)) + eps);
}
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// v into element i of array `arr` (shared memory) of every CTA of the cluster
__device__ __forceinline__ void store_to_cluster(float* arr, int i, float v) {
  const uint32_t local = static_cast<uint32_t>(__cvta_generic_to_shared(arr + i));
#pragma unroll
  for (int r = 0; r < kMlpCluster; ++r) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(r));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
  }
}

__global__ void __launch_bounds__(kMlpThreads) mlp1_kernel(const MlpArgs a) {
  SLMKV_TL(kTlMlp1);
  extern __shared__ __align__(16) uint8_t smem[];
  const int tid = threadIdx.x, H = a.H, I = a.I;
  const int CO = H / kMlpCluster, CI = I / kMlpCluster;
  const int HP = H + 8, IP = I + 8;  // padded row lengths (bank-conflict-free 16-byte loads)
  uint32_t rank;
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int o0 = static_cast<int>(rank) * CO, i0 = static_cast<int>(rank) * CI;
  const int CQ = a.wqkv ? (H + 2 * a.KV) / kMlpCluster : 0, q0 = static_cast<int>(rank) * CQ;
  uint16_t* wo_s = reinterpret_cast<uint16_t*>(smem);
  uint16_t* wg_s = wo_s + static_cast<size_t>(CO) * HP;
  uint16_t* wu_s = wg_s + static_cast<size_t>(CI) * HP;
  uint16_t* wd_s = wu_s + static_cast<size_t>(CI) * HP;
  uint16_t* wq_s = wd_s + static_cast<size_t>(CO) * IP;
  float* xo = reinterpret_cast<float*>(wq_s + static_cast<size_t>(CQ) * HP);
  float* hid = xo + H;
  float* xg = hid + H;
  float* hb = xg + H;
  float* up_s = hb + I;
  float* gf = up_s + CI;  // FFN norm scale
  float* ga = gf + H;     // the next layer's attention norm scale (with wqkv)
  __shared__ float inv_s;
  auto smem_u32 = [](const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); };
  // the weights and norm scales (no kernel writes them) are requested before
  // the wait, 16 bytes a copy along each output's row
  const int h8 = H / 8, i8 = I / 8;
  const uint16_t* wo = reinterpret_cast<const uint16_t*>(a.wo);
  const uint16_t* wgu = reinterpret_cast<const uint16_t*>(a.wgu);
  const uint16_t* wd = reinterpret_cast<const uint16_t*>(a.wd);
  const uint16_t* wq = reinterpret_cast<const uint16_t*>(a.wqkv);
  for (int i = tid; i < CO * h8; i += kMlpThreads) {
    const int j = i / h8, c = i - j * h8;
    cp_async16(smem_u32(wo_s + j * HP + 8 * c), wo + static_cast<size_t>(o0 + j) * H + 8 * c);
  }
  for (int i = tid; i < CI * h8; i += kMlpThreads) {
    const int j = i / h8, c = i - j * h8;
    cp_async16(smem_u32(wg_s + j * HP + 8 * c), wgu + static_cast<size_t>(i0 + j) * H + 8 * c);
    cp_async16(smem_u32(wu_s + j * HP + 8 * c), wgu + static_cast<size_t>(I + i0 + j) * H + 8 * c);
  }
  for (int i = tid; i < CO * i8; i += kMlpThreads) {
    const int j = i / i8, c = i - j * i8;
    cp_async16(smem_u32(wd_s + j * IP + 8 * c), wd + static_cast<size_t>(o0 + j) * I + 8 * c);
  }
  for (int i = tid; i < CQ * h8; i += kMlpThreads) {
    const int j = i / h8, c = i - j * h8;
    cp_async16(smem_u32(wq_s + j * HP + 8 * c), wq + static_cast<size_t>(q0 + j) * H + 8 * c);
  }
  for (int i = tid; i < H / 4; i += kMlpThreads) {
    cp_async16(smem_u32(gf + 4 * i), a.ffn_norm + 4 * i);
    if (a.wqkv) cp_async16(smem_u32(ga + 4 * i), a.attn_norm + 4 * i);
  }
  cp_async_commit();
  cluster_barrier();  // every CTA of the cluster runs before any writes another's shared memory
  wait_previous_kernel();  // the attention row comes from the previous kernel
  SLMKV_TL_MARK(kTlMlpPhase + 0);
  for (int k = tid; k < H; k += kMlpThreads) xo[k] = round_bf16(a.att[k]);  // the projection's operand
  float xres = 0.f;  // this thread's residual element
  if (tid < CO) xres = a.x[o0 + tid];
  cp_async_wait<0>();
  __syncthreads();
  SLMKV_TL_MARK(kTlMlpPhase + 1);
  // output projection, onto the residual (transformer.rs add_residual_in_place);
  // every CTA receives the new residual row
  if (tid < CO) {
    const float acc = fold_row(wo_s + tid * HP, xo, H);
    store_to_cluster(hid, o0 + tid, __fadd_rn(xres, acc));
  }
  cluster_barrier();
  SLMKV_TL_MARK(kTlMlpPhase + 2);
  // FFN RMSNorm (rmsnorm.rs:80-91)
  if (tid == 0) inv_s = inv_rms(hid, H, a.eps);
  __syncthreads();
  for (int k = tid; k < H; k += kMlpThreads) xg[k] = round_bf16(__fmul_rn(__fmul_rn(hid[k], inv_s), gf[k]));
  __syncthreads();
  SLMKV_TL_MARK(kTlMlpPhase + 3);
  // gate and up columns i0 .. i0 + CI, SiTU-GLU (situ_glu.rs:101-107) as bf16;
  // every CTA receives h
  float g = 0.f;
  if (tid < 2 * CI) {
    const int up = tid >= CI ? 1 : 0, cl = tid - up * CI;
    g = fold_row((up ? wu_s : wg_s) + cl * HP, xg, H);
    if (up) up_s[cl] = g;
  }
  __syncthreads();
  if (tid < CI)
    store_to_cluster(hb, i0 + tid,
                     round_bf16(__fmul_rn(situ_gate(g, a.beta_gate), situ_up(up_s[tid], a.beta_up))));
  cluster_barrier();
  SLMKV_TL_MARK(kTlMlpPhase + 4);
  // down projection, onto the residual
  if (tid < CO) {
    const float acc = fold_row(wd_s + tid * IP, hb, I);
    const float nx = __fadd_rn(hid[o0 + tid], acc);
    a.x[o0 + tid] = nx;
    if (a.wqkv) store_to_cluster(xo, o0 + tid, nx);  // xo is free: the next layer's row
  }
  if (!a.wqkv) return;
  cluster_barrier();
  SLMKV_TL_MARK(kTlMlpPhase + 5);
  // the next layer's attention RMSNorm and q/k/v columns q0 .. q0 + CQ
  if (tid == 0) inv_s = inv_rms(xo, H, a.eps);
  __syncthreads();
  for (int k = tid; k < H; k += kMlpThreads) xg[k] = round_bf16(__fmul_rn(__fmul_rn(xo[k], inv_s), ga[k]));
  __syncthreads();
  SLMKV_TL_MARK(kTlMlpPhase + 6);
  if (tid < CQ) {
    const int col = q0 + tid;
    const float acc = fold_row(wq_s + tid * HP, xg, H);
    if (col < H) a.q[col] = acc;
    else if (col < H + a.KV) a.k[col - H] = acc;
    else a.v[col - H - a.KV] = acc;
  }
}

cudaError_t launch_mlp1(const MlpArgs& a, cudaStream_t s) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(kMlpCluster);
  cfg.blockDim = dim3(kMlpThreads);
  cfg.dynamicSmemBytes = mlp1_smem(a.H, a.I, a.wqkv ? a.KV : 0);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = kMlpCluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, mlp1_kernel, a);
}

template <int MODE>
cudaError_t launch_proj(const ProjArgs& a, cudaStream_t s) {
  if (a.rows == 1 && a.cols > 0) {
    ProjArgs b = a;
    return launch_chained(proj1_kernel<MODE>, dim3((a.ncols + a.cols - 1) / a.cols),
                          dim3(proj_mats<MODE>() * a.cols), proj1_smem<MODE>(a.K, a.cols), s, b);
  }
  // several rows: the register-tiled kernel when its rows fit in shared
  // memory, 32-row tiles when they alone give two waves of CTAs, else 8-row
  constexpr size_t kSmemMax = 227 * 1024;
  if (a.rows > 1 && a.K % kPtChunk == 0 && a.ncols % 8 == 0) {
    const int cols = MODE == kProjGU ? kPtCols / 2 : kPtCols;
    const int64_t tiles4 = static_cast<int64_t>((a.rows + pt_rows(4) - 1) / pt_rows(4)) *
                           ((a.ncols + cols - 1) / cols);
    if (tiles4 >= 2 * 148 && projt_smem<4>(a.K) <= kSmemMax) return launch_projt_best<MODE, 4>(a, s, tiles4);
    const int64_t tiles1 = static_cast<int64_t>((a.rows + pt_rows(1) - 1) / pt_rows(1)) * ((a.ncols + cols - 1) / cols);
    if (projt_smem<1>(a.K) <= kSmemMax) return launch_projt_best<MODE, 1>(a, s, tiles1);
  }
  const int gx = (a.ncols + kProjCols - 1) / kProjCols;
  if (a.rows == 1)
    return launch_chained(proj_kernel<MODE, 1>, dim3(gx, 1), dim3(kProjThreads), proj_smem<MODE>(a.K), s, a);
  return launch_chained(proj_kernel<MODE, kProjRows>, dim3(gx, (a.rows + kProjRows - 1) / kProjRows),
                        dim3(kProjThreads), proj_smem<MODE>(a.K), s, a);
}

// The layers and the vocabulary projection for `rows` token rows of the
// open batch; `prefill` selects the append + prefill-attention cache step
// and projects only each sequence's last row. Up to kFusedRows rows the
// projections are the fused kernels above (5 launches a layer with the cache
// step); beyond, tensor-core GEMMs with separate norm / rounding / SiTU.
slm_status run_step(slm_model* m, slm_batch* b, const BatchRows& br, const int32_t* ids, int32_t rows,
                    bool prefill, float* logits, int32_t* next) {
  const int32_t out_rows = prefill ? br.n_seq : rows;
  slm_status rc = ensure_scratch(m, rows, out_rows, br.stream);
  if (rc) return rc;
  cudaStream_t s = br.stream;
  cublasStatus_t bs = cublasSetStream(m->blas, s);
  if (bs != CUBLAS_STATUS_SUCCESS) return blas_fail(m->ctx, "slm_model step", bs);
  int32_t* err = ctx_error_word(m->ctx);
  int32_t launches = 0;
  const int32_t H = m->H, I = m->I, KV = m->KV;
  const bool fused = rows <= m->exact_rows;
  // otherwise: few rows on the tensor-core row GEMMs, many on cuBLAS
  const bool row_gemms = !fused && rows <= kRowGemmRows;
  __nv_bfloat16* hb = reinterpret_cast<__nv_bfloat16*>(m->xb);
  // the fused path's kernels are chained (programmatic dependent launch)
  cudaError_t le = fused ? launch_chained(embed_kernel, dim3(rows), dim3(64), 0, s, ids, m->emb, m->V, H, m->x, err)
                         : (embed_kernel<<<rows, 64, 0, s>>>(ids, m->emb, m->V, H, m->x, err), cudaSuccess);
  ++launches;
  auto launched = [&](cudaError_t e2) {
    if (le == cudaSuccess) le = e2;
  };
  // The exact-order path on an f32 pool appends, then attends in the
  // reference's operation order (every score, the softmax sum and every
  // output fold as the CPU path computes them); otherwise the split-K decode
  // kernel or the prefill kernels.
  const bool exact_attention = fused && m->f32_pool;
  auto cache_step = [&](int32_t l) {
    if (prefill) {
      slm_status r = slm_batch_append_layer(b, l, m->k, m->v, 1);
      if (r) return r;
      return exact_attention ? slm_batch_attention_exact(b, l, m->q, 1, m->att)
                             : slm_batch_prefill_attention(b, l, m->q, 1, m->att);
    }
    return exact_attention ? slm_batch_decode_layer_exact(b, l, m->q, m->k, m->v, m->att)
                           : slm_batch_decode_layer(b, l, m->q, m->k, m->v, m->att);
  };
  bool qkv_done = false;  // the previous layer's cluster launch made this layer's q/k/v
  for (int32_t l = 0; l < m->L; ++l) {
    const slm_model::Layer& Ly = m->layers[l];
    if (fused) {
      ProjArgs a{};
      a.eps = m->eps;
      a.rows = rows;
      a.H = H;
      a.KV = KV;
      a.I = I;
      a.beta_gate = m->beta_gate;
      a.beta_up = m->beta_up;
      ProjArgs q = a;  // q, k, v with the attention RMSNorm
      q.x = m->x, q.norm_w = Ly.attn_norm, q.K = H, q.ncols = H + 2 * KV, q.w = Ly.wqkv, q.ld = H + 2 * KV;
      q.cols = m->p1_cols[kProjQKV];
      q.y0 = m->q, q.y1 = m->k, q.y2 = m->v;
      if (!qkv_done) {
        launched(launch_proj<kProjQKV>(q, s));
        ++launches;
      }
      qkv_done = false;
      if ((rc = cache_step(l))) return rc;
      if (rows == 1 && m->mlp1_ok) {
        // output, FFN norm, gate/up, down (and the next layer's norm and
        // q/k/v): one cluster launch
        MlpArgs ma{m->att, m->x, Ly.wo_r, Ly.wgu_r, Ly.wd_r, Ly.ffn_norm, m->eps,
                   m->beta_gate, m->beta_up, H, I};
        if (l + 1 < m->L && m->mlp1_qkv_ok) {
          ma.wqkv = m->layers[l + 1].wqkv_r;
          ma.attn_norm = m->layers[l + 1].attn_norm;
          ma.q = m->q;
          ma.k = m->k;
          ma.v = m->v;
          ma.KV = KV;
          qkv_done = true;
        }
        launched(launch_mlp1(ma, s));
        ++launches;
        continue;
      }
      ProjArgs o = a;  // output projection onto the residual
      o.x = m->att, o.K = H, o.ncols = H, o.w = Ly.wo, o.ld = H, o.y0 = m->x;
      o.cols = m->p1_cols[kProjO];
      launched(launch_proj<kProjO>(o, s));
      ProjArgs g = a;  // gate / up with the FFN RMSNorm, SiTU-GLU
      g.x = m->x, g.norm_w = Ly.ffn_norm, g.K = H, g.ncols = I, g.w = Ly.wgu, g.ld = 2 * I, g.h = hb;
      g.cols = m->p1_cols[kProjGU];
      launched(launch_proj<kProjGU>(g, s));
      ProjArgs d = a;  // down projection onto the residual
      d.xh = hb, d.K = I, d.ncols = H, d.w = Ly.wd, d.ld = H, d.y0 = m->x;
      d.cols = m->p1_cols[kProjDown];
      launched(launch_proj<kProjDown>(d, s));
      launches += 3;
      continue;
    }
    const int32_t nqkv = H + 2 * KV;
    if (row_gemms) {
      // tensor-core row GEMMs (slmkv_rowgemm.cu), every kernel chained
      RowGemmLaunch a{};
      a.rows = rows;
      a.H = H;
      a.KV = KV;
      a.I = I;
      a.beta_gate = m->beta_gate;
      a.beta_up = m->beta_up;
      a.err = err;
      auto gemm = [&](int mode, const CUtensorMap& tw, const void* x, int32_t K, int32_t ncols) -> slm_status {
        const RowGemmPlan q = plan_row_gemm(mode, rows, K, ncols, m->sms);
        RowGemmLaunch g = a;
        g.tmap_w = tw;
        g.x = x;
        g.K = K;
        g.ncols = ncols;
        const cudaError_t e2 = launch_row_gemm(mode, g, q, s);
        if (e2 != cudaSuccess) return cuda_fail(m->ctx, "slm_model row GEMM", e2);
        ++launches;
        return SLM_OK;
      };
      // The RMSNorms run across the projections (slmkv_rowgemm.cu): the
      // previous residual update wrote bf16(x * g) and its square sums,
      // q/k/v and gate/up scale by 1 / rms. The first layer's attention
      // norm, after the embedding, is a kernel of its own.
      a.ssq_ld = ssq_tiles(H);
      a.eps = m->eps;
      a.y0 = m->q, a.y1 = m->k, a.y2 = m->v;
      if (l == 0) {
        launched(launch_chained(rmsnorm_kernel, dim3(rows), dim3(kNormThreads), 0, s,
                                static_cast<const float*>(m->x), rows, H, Ly.attn_norm, m->eps, m->xb,
                                static_cast<float*>(nullptr), static_cast<const SeqEntry*>(nullptr),
                                static_cast<uint32_t*>(nullptr)));
        ++launches;
        if ((rc = gemm(kRowQKV, Ly.tm_qkv, m->xb, H, nqkv))) return rc;
      } else {
        a.ssq_in = m->ssq;
        rc = gemm(kRowQKV, Ly.tm_qkv, m->xg, H, nqkv);
        a.ssq_in = nullptr;
        if (rc) return rc;
      }
      if (!prefill && !exact_attention) {
        // the decode kernel also writes the attention rows rounded to bf16,
        // the output projection's operand (no separate rounding launch)
        if ((rc = batch_decode_layer_bf16(b, l, m->q, m->k, m->v, m->att,
                                          reinterpret_cast<uint32_t*>(m->xb))))
          return rc;
      } else {
        if ((rc = cache_step(l))) return rc;
        const size_t n4 = static_cast<size_t>(rows) * H / 4;
        launched(launch_chained(round_bf16_kernel, dim3(grid_for(n4, 256)), dim3(256), 0, s,
                                reinterpret_cast<const float4*>(m->att), n4,
                                reinterpret_cast<uint2*>(m->xb)));
        ++launches;
      }
      a.y0 = m->x, a.y1 = a.y2 = nullptr;
      a.xg = m->xg, a.ssq = m->ssq;
      a.norm_next = Ly.ffn_norm;
      if ((rc = gemm(kRowO, Ly.tm_o, m->xb, H, H))) return rc;
      a.norm_next = nullptr;
      a.h = m->hb;
      a.ssq_in = m->ssq;
      if ((rc = gemm(kRowGU, Ly.tm_gu, m->xg, H, I))) return rc;
      a.ssq_in = nullptr;
      a.norm_next = l + 1 < m->L ? m->layers[l + 1].attn_norm : nullptr;
      if ((rc = gemm(kRowDown, Ly.tm_d, m->hb, I, H))) return rc;
      continue;
    }
    rmsnorm_kernel<<<rows, kNormThreads, 0, s>>>(m->x, rows, H, Ly.attn_norm, m->eps, m->xb, nullptr, nullptr);
    ++launches;
    if ((bs = gemm_t(m->blas, m->xb, rows, H, Ly.wqkv, nqkv, H, m->q, 0.f)) != CUBLAS_STATUS_SUCCESS ||
        (bs = gemm_t(m->blas, m->xb, rows, H, Ly.wqkv + H, nqkv, KV, m->k, 0.f)) != CUBLAS_STATUS_SUCCESS ||
        (bs = gemm_t(m->blas, m->xb, rows, H, Ly.wqkv + H + KV, nqkv, KV, m->v, 0.f)) !=
            CUBLAS_STATUS_SUCCESS)
      return blas_fail(m->ctx, "slm_model q/k/v projection", bs);
    if ((rc = cache_step(l))) return rc;
    const size_t n4 = static_cast<size_t>(rows) * H / 4;
    round_bf16_kernel<<<grid_for(n4, 256), 256, 0, s>>>(reinterpret_cast<const float4*>(m->att), n4,
                                                         reinterpret_cast<uint2*>(m->xb));
    ++launches;
    if ((bs = gemm_t(m->blas, m->xb, rows, H, Ly.wo, H, H, m->x, 1.f)) != CUBLAS_STATUS_SUCCESS)
      return blas_fail(m->ctx, "slm_model output projection", bs);
    rmsnorm_kernel<<<rows, kNormThreads, 0, s>>>(m->x, rows, H, Ly.ffn_norm, m->eps, m->xb, nullptr, nullptr);
    ++launches;
    if ((bs = gemm_t(m->blas, m->xb, rows, H, Ly.wgu, 2 * I, 2 * I, m->gu, 0.f)) != CUBLAS_STATUS_SUCCESS)
      return blas_fail(m->ctx, "slm_model gate/up projection", bs);
    const size_t pairs = static_cast<size_t>(rows) * (I / 2);
    situ_kernel<<<grid_for(pairs, 256), 256, 0, s>>>(m->gu, rows, I, m->beta_gate, m->beta_up, m->xb);
    ++launches;
    if ((bs = gemm_t(m->blas, m->xb, rows, I, Ly.wd, H, H, m->x, 1.f)) != CUBLAS_STATUS_SUCCESS)
      return blas_fail(m->ctx, "slm_model down projection", bs);
  }
  if (logits || next) {
    const SeqEntry* last_rows = prefill ? br.d_seqs : nullptr;
    // the row-GEMM path's head: tensor cores over the split operands
    const bool head3 = !fused && m->head3 != nullptr && out_rows <= kRowGemmRows;
    if (fused)
      launched(launch_chained(rmsnorm_kernel, dim3(out_rows), dim3(kNormThreads), 0, s, m->x, out_rows, H,
                              m->final_norm, m->eps, static_cast<uint32_t*>(nullptr), m->xf, last_rows,
                              static_cast<uint32_t*>(nullptr)));
    else
      rmsnorm_kernel<<<out_rows, kNormThreads, 0, s>>>(m->x, out_rows, H, m->final_norm, m->eps, nullptr,
                                                       m->xf, last_rows, head3 ? m->xs3 : nullptr);
    ++launches;
    float* lg = logits ? logits : m->logits;
    if (head3) {
      RowGemmLaunch g{};
      g.rows = out_rows;
      g.H = H;
      g.KV = KV;
      g.I = I;
      g.err = err;
      g.tmap_w = m->tm_head;
      g.x = m->xs3;
      g.K = 3 * H;
      g.ncols = m->V;
      g.y0 = lg;
      const RowGemmPlan q = plan_row_gemm(kRowHead, out_rows, 3 * H, m->V, m->sms);
      const cudaError_t e2 = launch_row_gemm(kRowHead, g, q, s);
      if (e2 != cudaSuccess) return cuda_fail(m->ctx, "slm_model vocabulary projection", e2);
      ++launches;
    } else if (out_rows > 1 && out_rows <= kHeadMaxRows && m->head_kernel_ok) {
      const dim3 grid((m->V + kHeadEntries - 1) / kHeadEntries, (out_rows + kHeadRows - 1) / kHeadRows);
      launched(launch_chained(head_kernel, grid, dim3(kHeadThreads), static_cast<size_t>(kHeadRows) * H * 4, s,
                              static_cast<const float*>(m->xf), out_rows, H, m->emb, m->V, lg));
      ++launches;
    } else {
      const float one = 1.f, zero = 0.f;
      bs = cublasSgemm(m->blas, CUBLAS_OP_T, CUBLAS_OP_N, m->V, out_rows, H, &one, m->emb, H, m->xf, H, &zero,
                       lg, m->V);
      if (bs != CUBLAS_STATUS_SUCCESS) return blas_fail(m->ctx, "slm_model vocabulary projection", bs);
    }
    if (next) {
      launched(launch_chained(argmax_kernel, dim3(out_rows), dim3(kArgmaxThreads), 0, s,
                              static_cast<const float*>(lg), m->V, next, err));
      ++launches;
    }
  }
  ctx_count_launches(m->ctx, launches);
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(m->ctx, "slm_model step", e);
  return SLM_OK;
}

}  // namespace
SLMKV_TL_SETTER(timeline_set_model)

}  // namespace slmkv

using namespace slmkv;

extern "C" {

slm_status slm_model_create(slm_ctx* ctx, const slm_model_config* config, const float* const* h_tensors,
                            int32_t n_tensors, slm_model** out) {
  if (!ctx || !config || !h_tensors || !out) return SLM_ERR_INVALID_INPUT;
  *out = nullptr;
  slm_config c{};
  slm_status rc = slm_ctx_config(ctx, &c);
  if (rc) return rc;
  if ((rc = ctx_need_device(ctx))) return rc;
  const int32_t V = config->vocab_size, H = config->hidden_size, I = config->intermediate_size;
  const int32_t L = c.num_layers, KV = c.num_key_value_heads * c.head_dimension;
  // config.rs:91-198 (the parts the device path relies on)
  if (V <= 0 || H != c.num_query_heads * c.head_dimension || H > kNormMaxWidth || I <= 0 || I % 8 != 0)
    return ctx_fail(ctx, SLM_ERR_INVALID_CONFIGURATION,
                    "invalid model configuration: vocab > 0, hidden = query heads x head dimension "
                    "(at most 8192), intermediate a positive multiple of 8");
  if (!(config->rms_norm_epsilon > 0.f) || !std::isfinite(config->rms_norm_epsilon) ||
      !std::isfinite(config->situ_beta_gate) || !std::isfinite(config->situ_beta_up) ||
      config->situ_beta_gate == 0.f || config->situ_beta_up == 0.f)
    return ctx_fail(ctx, SLM_ERR_INVALID_CONFIGURATION,
                    "invalid model configuration: rms_norm_epsilon finite and > 0, SiTU betas finite "
                    "and non-zero");
  if (n_tensors != 2 + 9 * L)
    return ctx_fail(ctx, SLM_ERR_INVALID_INPUT, "invalid input for model weights: 2 + 9 * layers tensors");
  for (int32_t i = 0; i < n_tensors; ++i)
    if (!h_tensors[i]) return ctx_fail(ctx, SLM_ERR_INVALID_INPUT, "invalid input for model weights: null tensor");

  // One host image of the device allocation: fp32 embedding and norms,
  // bf16 projection matrices ([gate; up] concatenated), 256-byte aligned.
  const size_t HH = static_cast<size_t>(H) * H, KH = static_cast<size_t>(KV) * H,
               IH = static_cast<size_t>(I) * H;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t o_emb = take(static_cast<size_t>(V) * H * 4), o_final = take(static_cast<size_t>(H) * 4);
  struct LayerOff {
    size_t an, fn, qkv, o, gu, d;
    size_t qkv_r, o_r, gu_r, d_r;  // [out][in] copies for the one-row cluster launch
  };
  const bool rows_out = mlp1_fits(H, I, 0);
  std::vector<LayerOff> lo(static_cast<size_t>(L));
  for (auto& x : lo) {
    x.an = take(static_cast<size_t>(H) * 4);
    x.fn = take(static_cast<size_t>(H) * 4);
    x.qkv = take((HH + 2 * KH) * 2);
    x.o = take(HH * 2);
    x.gu = take(2 * IH * 2);
    x.d = take(IH * 2);
    if (rows_out) {
      x.qkv_r = take((HH + 2 * KH) * 2);
      x.o_r = take(HH * 2);
      x.gu_r = take(2 * IH * 2);
      x.d_r = take(IH * 2);
    }
  }
  std::vector<uint8_t> img(off);
  auto put_f32 = [&](size_t o, const float* src, size_t n) { std::memcpy(img.data() + o, src, n * 4); };
  // src [rows][cols] (the reference's [out][in]) into columns [col0, col0 +
  // rows) of a transposed [cols][ld] bf16 matrix at byte offset o
  auto put_bf16_t = [&](size_t o, const float* src, int32_t rows, int32_t cols, int32_t ld,
                        int32_t col0) {
    uint16_t* d = reinterpret_cast<uint16_t*>(img.data() + o);
    for (int32_t r = 0; r < rows; ++r)
      for (int32_t c2 = 0; c2 < cols; ++c2)
        d[static_cast<size_t>(c2) * ld + col0 + r] = bf16_bits(src[static_cast<size_t>(r) * cols + c2]);
  };
  // src [rows][cols] as bf16 rows at byte offset o (the reference's layout)
  auto put_bf16 = [&](size_t o, const float* src, size_t n) {
    uint16_t* d = reinterpret_cast<uint16_t*>(img.data() + o);
    for (size_t i = 0; i < n; ++i) d[i] = bf16_bits(src[i]);
  };
  put_f32(o_emb, h_tensors[0], static_cast<size_t>(V) * H);
  put_f32(o_final, h_tensors[1 + 9 * L], static_cast<size_t>(H));
  for (int32_t l = 0; l < L; ++l) {
    const float* const* t = h_tensors + 1 + 9 * l;
    const LayerOff& x = lo[static_cast<size_t>(l)];
    const int32_t nqkv = H + 2 * KV;
    put_f32(x.an, t[0], static_cast<size_t>(H));
    put_bf16_t(x.qkv, t[1], H, H, nqkv, 0);
    put_bf16_t(x.qkv, t[2], KV, H, nqkv, H);
    put_bf16_t(x.qkv, t[3], KV, H, nqkv, H + KV);
    put_bf16_t(x.o, t[4], H, H, H, 0);
    put_f32(x.fn, t[5], static_cast<size_t>(H));
    put_bf16_t(x.gu, t[6], I, H, 2 * I, 0);  // gate columns first
    put_bf16_t(x.gu, t[7], I, H, 2 * I, I);  // then up
    put_bf16_t(x.d, t[8], H, I, H, 0);
    if (rows_out) {
      put_bf16(x.qkv_r, t[1], HH);
      put_bf16(x.qkv_r + HH * 2, t[2], KH);
      put_bf16(x.qkv_r + (HH + KH) * 2, t[3], KH);
      put_bf16(x.o_r, t[4], HH);
      put_bf16(x.gu_r, t[6], IH);
      put_bf16(x.gu_r + IH * 2, t[7], IH);
      put_bf16(x.d_r, t[8], IH);
    }
  }
  auto m = new slm_model();
  m->ctx = ctx;
  m->f32_pool = c.kv_dtype == SLM_KV_F32;
  m->V = V;
  m->H = H;
  m->I = I;
  m->L = L;
  m->KV = KV;
  m->eps = config->rms_norm_epsilon;
  m->beta_gate = config->situ_beta_gate;
  m->beta_up = config->situ_beta_up;
  cudaError_t e = cudaMalloc(&m->weights, off);
  if (e == cudaSuccess) e = cudaMemcpy(m->weights, img.data(), off, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    slm_model_destroy(m);
    return cuda_fail(ctx, "slm_model_create", e);
  }
  const cublasStatus_t bs = cublasCreate(&m->blas);
  if (bs != CUBLAS_STATUS_SUCCESS) {
    m->blas = nullptr;
    slm_model_destroy(m);
    return blas_fail(ctx, "slm_model_create", bs);
  }
  cublasSetMathMode(m->blas, CUBLAS_DEFAULT_MATH);  // fp32 SGEMM without TF32
  // the fused projections stage kProjRows input rows and the weight ring;
  // a model whose rows do not fit runs every step on the GEMM path
  int dev = 0, optin = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) {
    slm_model_destroy(m);
    return cuda_fail(ctx, "slm_model_create", e);
  }
  m->exact_fits = std::max({proj_smem<kProjQKV>(H), proj_smem<kProjO>(H), proj_smem<kProjGU>(H),
                            proj_smem<kProjDown>(I)}) <= static_cast<size_t>(optin);
  m->exact_rows = m->exact_fits ? kFusedRows : 0;
  if (m->exact_fits) {
    auto attr = [&](auto kernel, size_t bytes) {
      return bytes > 48 * 1024 ? cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                      static_cast<int>(bytes))
                               : cudaSuccess;
    };
    cudaError_t a = attr(proj_kernel<kProjQKV, 1>, proj_smem<kProjQKV>(H));
    if (a == cudaSuccess) a = attr(proj_kernel<kProjO, 1>, proj_smem<kProjO>(H));
    if (a == cudaSuccess) a = attr(proj_kernel<kProjGU, 1>, proj_smem<kProjGU>(H));
    if (a == cudaSuccess) a = attr(proj_kernel<kProjDown, 1>, proj_smem<kProjDown>(I));
    if (a == cudaSuccess) a = attr(proj_kernel<kProjQKV, kProjRows>, proj_smem<kProjQKV>(H));
    if (a == cudaSuccess) a = attr(proj_kernel<kProjO, kProjRows>, proj_smem<kProjO>(H));
    if (a == cudaSuccess) a = attr(proj_kernel<kProjGU, kProjRows>, proj_smem<kProjGU>(H));
    if (a == cudaSuccess) a = attr(proj_kernel<kProjDown, kProjRows>, proj_smem<kProjDown>(I));
    if (a != cudaSuccess) {
      slm_model_destroy(m);
      return cuda_fail(ctx, "slm_model_create", a);
    }
    auto one_row = [&](auto kernel, int32_t cols, size_t bytes, int mode) {
      if (cols > 0 && attr(kernel, bytes) == cudaSuccess) m->p1_cols[mode] = cols;
    };
    one_row(proj1_kernel<kProjQKV>, proj1_cols<kProjQKV>(H), proj1_smem<kProjQKV>(H, proj1_cols<kProjQKV>(H)), kProjQKV);
    one_row(proj1_kernel<kProjO>, proj1_cols<kProjO>(H), proj1_smem<kProjO>(H, proj1_cols<kProjO>(H)), kProjO);
    one_row(proj1_kernel<kProjGU>, proj1_cols<kProjGU>(H), proj1_smem<kProjGU>(H, proj1_cols<kProjGU>(H)), kProjGU);
    one_row(proj1_kernel<kProjDown>, proj1_cols<kProjDown>(I), proj1_smem<kProjDown>(I, proj1_cols<kProjDown>(I)),
            kProjDown);
    m->mlp1_qkv_ok = rows_out && mlp1_fits(H, I, KV) && attr(mlp1_kernel, mlp1_smem(H, I, KV)) == cudaSuccess;
    m->mlp1_ok = m->mlp1_qkv_ok ||
                 (rows_out && attr(mlp1_kernel, mlp1_smem(H, I, 0)) == cudaSuccess);
  }
  const uint8_t* base = static_cast<const uint8_t*>(m->weights);
  m->emb = reinterpret_cast<const float*>(base + o_emb);
  m->final_norm = reinterpret_cast<const float*>(base + o_final);
  if (H <= kHeadMaxWidth) {
    e = cudaFuncSetAttribute(head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kHeadRows * H * 4);
    if (e != cudaSuccess) {
      slm_model_destroy(m);
      return cuda_fail(ctx, "slm_model_create", e);
    }
    m->head_kernel_ok = true;
  }
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) {
    slm_model_destroy(m);
    return cuda_fail(ctx, "slm_model_create", e);
  }
  m->sms = sms;
  for (const LayerOff& x : lo) {
    auto bf = [&](size_t o) { return reinterpret_cast<const __nv_bfloat16*>(base + o); };
    slm_model::Layer Ly{};
    Ly.attn_norm = reinterpret_cast<const float*>(base + x.an);
    Ly.ffn_norm = reinterpret_cast<const float*>(base + x.fn);
    Ly.wqkv = bf(x.qkv);
    Ly.wo = bf(x.o);
    Ly.wgu = bf(x.gu);
    Ly.wd = bf(x.d);
    if (rows_out) {
      Ly.wqkv_r = bf(x.qkv_r);
      Ly.wo_r = bf(x.o_r);
      Ly.wgu_r = bf(x.gu_r);
      Ly.wd_r = bf(x.d_r);
    }
    // [K rows][columns] bf16, 64 x 64 boxes
    const int32_t nqkv = H + 2 * KV;
    e = encode_row_gemm_map(&Ly.tm_qkv, Ly.wqkv, nqkv, H, 64, 64);
    if (e == cudaSuccess) e = encode_row_gemm_map(&Ly.tm_o, Ly.wo, H, H, 64, 64);
    if (e == cudaSuccess) e = encode_row_gemm_map(&Ly.tm_gu, Ly.wgu, 2 * I, H, 64, 64);
    if (e == cudaSuccess) e = encode_row_gemm_map(&Ly.tm_d, Ly.wd, H, I, 64, 64);
    if (e != cudaSuccess) {
      slm_model_destroy(m);
      return cuda_fail(ctx, "slm_model_create (weight tensor maps)", e);
    }
    m->layers.push_back(Ly);
  }
  // the row-GEMM path's tied head as one split-bf16 GEMM (hidden >= 512)
  if (H >= 512 && H % 64 == 0 && V % 8 == 0) {
    const size_t n = static_cast<size_t>(2) * H * V;
    e = cudaMalloc(&m->head3, n * 2);
    if (e == cudaSuccess) {
      head_split_kernel<<<dim3((V + 31) / 32, (H + 31) / 32), dim3(32, 8)>>>(m->emb, V, H, m->head3);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = encode_row_gemm_map(&m->tm_head, m->head3, V, 2 * H, 64, 64);
    if (e != cudaSuccess) {
      slm_model_destroy(m);
      return cuda_fail(ctx, "slm_model_create (split head)", e);
    }
  }
  *out = m;
  return SLM_OK;
}

slm_status slm_model_set_exact_rows(slm_model* m, int32_t max_rows) {
  if (!m) return SLM_ERR_INVALID_INPUT;
  if (max_rows < 0 || max_rows > kFusedRows)
    return ctx_fail(m->ctx, SLM_ERR_INVALID_INPUT,
                    "invalid input for model projections: exact-order rows must be in [0, 1024]");
  if (max_rows > 0 && !m->exact_fits)
    return ctx_fail(m->ctx, SLM_ERR_INVALID_INPUT,
                    "invalid input for model projections: this model's rows do not fit the exact-order "
                    "kernels' shared memory");
  m->exact_rows = max_rows;
  return SLM_OK;
}

slm_status slm_model_destroy(slm_model* m) {
  if (!m) return SLM_ERR_INVALID_INPUT;
  free_scratch(m);
  if (m->weights) cudaFree(m->weights);
  if (m->head3) cudaFree(m->head3);
  if (m->blas) cublasDestroy(m->blas);
  delete m;
  return SLM_OK;
}

slm_status slm_model_decode(slm_model* m, slm_batch* b, const int32_t* d_token_ids, float* d_logits,
                            int32_t* d_next_token) {
  if (!m || !b || !d_token_ids) return SLM_ERR_INVALID_INPUT;
  if (batch_ctx(b) != m->ctx)
    return ctx_fail(m->ctx, SLM_ERR_INVALID_INPUT, "invalid input for model step: batch of another context");
  slm_status rc = ctx_need_device(m->ctx);
  if (rc) return rc;
  const BatchRows br = batch_rows(b);
  for (int32_t i = 0; i < br.n_seq; ++i)
    if (br.counts[i] != 1)
      return ctx_fail(m->ctx, SLM_ERR_INVALID_INPUT,
                      "invalid input for model cached decode: one token per sequence (model.rs:342)");
  if (br.n_seq == 0) return SLM_OK;
  return run_step(m, b, br, d_token_ids, br.n_seq, false, d_logits, d_next_token);
}

slm_status slm_model_prefill(slm_model* m, slm_batch* b, const int32_t* d_token_ids, float* d_logits,
                             int32_t* d_next_token) {
  if (!m || !b || !d_token_ids) return SLM_ERR_INVALID_INPUT;
  if (batch_ctx(b) != m->ctx)
    return ctx_fail(m->ctx, SLM_ERR_INVALID_INPUT, "invalid input for model step: batch of another context");
  slm_status rc = ctx_need_device(m->ctx);
  if (rc) return rc;
  const BatchRows br = batch_rows(b);
  if (br.n_seq == 0 || br.total_tokens == 0) return SLM_OK;
  return run_step(m, b, br, d_token_ids, br.total_tokens, true, d_logits, d_next_token);
}

}  // extern "C"
