// Live kernel timeline for profiling builds only
// (make EXTRA_NVFLAGS=-DSLMKV_TIMELINE; compiled out otherwise).
//
// ncu serializes the launches it measures, so it cannot show how the chained
// kernels of a step (programmatic dependent launch) overlap on the GPU. In a
// timeline build every warp of an instrumented kernel records its kernel
// kind, CTA, SM and %globaltimer at entry and exit into a device buffer that
// the host hands over with slmkv_timeline_set (exported, not part of the
// public header), one record per warp.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace slmkv {

struct TimelineRec {
  uint16_t kind;   // TimelineKind
  uint16_t sm;     // %smid
  uint32_t block;  // blockIdx.x | blockIdx.y << 16 (low bits)
  uint64_t t0, t1; // %globaltimer (ns) at entry and exit
};
static_assert(sizeof(TimelineRec) == 24, "timeline record layout");

enum TimelineKind : uint16_t {
  kTlDecode = 1, kTlDecodeLayers, kTlAppend, kTlGather, kTlPrefill, kTlExact, kTlApply,
  kTlEmbed, kTlNorm, kTlRound, kTlSitu, kTlProj, kTlHead, kTlArgmax, kTlProj1, kTlPrefillTc,
  kTlMlp1,
  kTlDecodeWaited = 24,    // a decode warp passed its wait on the previous kernel
  kTlDecodeSliceDone = 25, // a decode warp's slice streamed, its in-CTA merges done
  kTlExactWaited = 26,     // exact attention: past the wait on the previous kernel
  kTlExactSoftmax = 27,    // exact attention: probabilities ready, value folds start
  kTlExactScored = 28,     // exact attention: scores and their maximum
  kTlExactSummed = 29,     // exact attention: the softmax sum
  kTlExactFolded = 30,     // exact attention: a folding warp's outputs stored
  kTlRowGemm = 32,      // + the row GEMM's mode
  kTlRowGemmMmaDone = 40,  // + mode: a CTA's MMAs complete (its epilogue starts)
  kTlRowGemmWaited = 48,   // + mode: the producer passed the wait on the previous kernel
  kTlMlpPhase = 56,        // + 0..6: a one-row cluster launch's phase boundaries
  kTlRowGemmPartials = 64, // + mode: the cluster's partial sums in shared memory
  kTlRowGemmStored = 72,   // + mode: a CTA's epilogue stores issued
};

#ifdef SLMKV_TIMELINE
namespace {
__device__ TimelineRec* g_tl_buf;
__device__ unsigned* g_tl_count;
__device__ unsigned g_tl_cap;

struct TlScope {
  uint16_t kind;
  uint64_t t0;
  __device__ explicit TlScope(uint16_t k) : kind(k) {
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  }
  __device__ ~TlScope() {
    if ((threadIdx.x & 31) != 0 || g_tl_buf == nullptr) return;
    uint64_t t1;
    uint32_t sm;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    const unsigned i = atomicAdd(g_tl_count, 1u);
    if (i < g_tl_cap)
      g_tl_buf[i] = TimelineRec{kind, static_cast<uint16_t>(sm),
                                (blockIdx.x & 0xffffu) | (blockIdx.y << 16), t0, t1};
  }
};

// A point event (t0 = t1 = now) from lane 0 of the calling warp.
__device__ __forceinline__ void tl_mark(uint16_t kind) {
  if ((threadIdx.x & 31) != 0 || g_tl_buf == nullptr) return;
  uint64_t t;
  uint32_t sm;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
  const unsigned i = atomicAdd(g_tl_count, 1u);
  if (i < g_tl_cap)
    g_tl_buf[i] = TimelineRec{kind, static_cast<uint16_t>(sm),
                              (blockIdx.x & 0xffffu) | (blockIdx.y << 16), t, t};
}

// Points this translation unit's kernels at the buffer (null: off).
inline cudaError_t timeline_set_here(TimelineRec* buf, unsigned* count, unsigned cap) {
  cudaError_t e = cudaMemcpyToSymbol(g_tl_buf, &buf, sizeof buf);
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_tl_count, &count, sizeof count);
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_tl_cap, &cap, sizeof cap);
  return e;
}
}  // namespace

// one per translation unit with instrumented kernels
cudaError_t timeline_set_kernels(TimelineRec* buf, unsigned* count, unsigned cap);
cudaError_t timeline_set_model(TimelineRec* buf, unsigned* count, unsigned cap);
cudaError_t timeline_set_rowgemm(TimelineRec* buf, unsigned* count, unsigned cap);
cudaError_t timeline_set_prefill_tc(TimelineRec* buf, unsigned* count, unsigned cap);

#define SLMKV_TL(kind) ::slmkv::TlScope slmkv_tl_scope_(kind)
#define SLMKV_TL_MARK(kind) ::slmkv::tl_mark(kind)
#define SLMKV_TL_SETTER(name)                                                              \
  cudaError_t name(TimelineRec* buf, unsigned* count, unsigned cap) {                     \
    return timeline_set_here(buf, count, cap);                                            \
  }
#else
#define SLMKV_TL(kind) ((void)0)
#define SLMKV_TL_MARK(kind) ((void)0)
#define SLMKV_TL_SETTER(name)
#endif

}  // namespace slmkv
