// Decode plan builder shared by the context path (slmkv_host.cpp) and the
// allocation-free entry point (slmkv_noalloc.cu). Host code only.
#pragma once

#include <algorithm>
#include <cstdint>

#include "slmkv_internal.h"

namespace slmkv {

// Sizes of a plan for n sequences attending ctx_len[i] tokens each.
struct PlanSizes {
  int64_t n_pairs = 0;    // n * kv_heads
  int64_t n_chunks = 0;   // stream length: sum over pairs of ceil(ctx_len / 16)
  int32_t n_warps = 0;    // decode warps used: min(available, n_chunks)
};

inline PlanSizes plan_sizes(int32_t n, const int32_t* ctx_len, int32_t kv_heads,
                            int32_t warps_available) {
  PlanSizes s;
  s.n_pairs = static_cast<int64_t>(n) * kv_heads;
  int64_t blocks = 0;
  for (int32_t i = 0; i < n; ++i) blocks += (ctx_len[i] + kBlockTokens - 1) / kBlockTokens;
  s.n_chunks = blocks * kv_heads;
  s.n_warps = static_cast<int32_t>(std::min<int64_t>(warps_available, s.n_chunks));
  return s;
}

// Builds the decode plan into caller-sized arrays (sizes from plan_sizes):
//   pairs[n_pairs]        one PairEntry per (row, KV head) in row order
//   chunks[n_chunks]      the stream: chunk = physical block * kv_heads + head
//   warp_start[2*n_warps] {first pair, seq, head, ctx_len}, {first pair's end, g0, g1, 0}
//   bounds[n_warps + 1]   scratch: warp w owns stream [bounds[w], bounds[w+1])
// block_of(i, j) is the physical block of row i's logical block j.
// Returns the number of cross-CTA partial slots the plan uses. Warp
// boundaries are floor(w*T/NW), stepped without divisions, and matched to
// pairs in one forward sweep.
template <typename BlockOf>
int32_t build_decode_plan(int32_t n, const int32_t* ctx_len, BlockOf block_of, int32_t kv_heads,
                          int32_t warps_per_cta, const PlanSizes& sz, PairEntry* pairs,
                          int32_t* chunks, int4* warp_start, int32_t* bounds) {
  int32_t cursor = 0, pi = 0;
  for (int32_t i = 0; i < n; ++i) {
    const int32_t nb = (ctx_len[i] + kBlockTokens - 1) / kBlockTokens;
    for (int32_t h = 0; h < kv_heads; ++h) {
      PairEntry pe{};
      pe.seq = i;
      pe.head = h;
      pe.ctx_len = ctx_len[i];
      pe.blk_begin = cursor;
      pe.nblk = nb;
      pairs[pi++] = pe;
      for (int32_t j = 0; j < nb; ++j) chunks[cursor++] = block_of(i, j) * kv_heads + h;
    }
  }
  const int64_t T = sz.n_chunks;
  const int32_t NW = sz.n_warps;
  {
    const int64_t q = T / NW, r = T % NW;
    int64_t b = 0, carry = 0;
    bounds[0] = 0;
    for (int32_t w = 0; w < NW; ++w) {
      carry += r;
      b += q;
      if (carry >= NW) {
        carry -= NW;
        ++b;
      }
      bounds[w + 1] = static_cast<int32_t>(b);
    }
  }
  int32_t wa = 0, wb = 0, part = 0;
  for (int64_t k = 0; k < sz.n_pairs; ++k) {
    PairEntry& pe = pairs[k];
    while (bounds[wa + 1] <= pe.blk_begin) ++wa;
    const int32_t last = pe.blk_begin + pe.nblk - 1;
    if (wb < wa) wb = wa;
    while (bounds[wb + 1] <= last) ++wb;
    pe.first_warp = wa;
    pe.nseg = wb - wa + 1;
    if (bounds[wa] == pe.blk_begin) pe.nseg |= (1 << 30);
    pe.part_base = part;
    // Pairs merge per CTA first (warps_per_cta consecutive warps); a pair
    // that spans CTAs takes one global partial slot per CTA it touches.
    const int32_t n_cta = wb / warps_per_cta - wa / warps_per_cta + 1;
    if (n_cta > 1) part += n_cta;
  }
  int64_t pc = 0;
  for (int32_t w = 0; w < NW; ++w) {
    const int32_t b = bounds[w];
    while (pairs[pc].blk_begin + pairs[pc].nblk <= b) ++pc;
    const PairEntry& pe = pairs[pc];
    warp_start[2 * w] = make_int4(static_cast<int32_t>(pc), pe.seq, pe.head, pe.ctx_len);
    warp_start[2 * w + 1] = make_int4(pe.blk_begin + pe.nblk, b, bounds[w + 1], 0);
  }
  return part;
}

}  // namespace slmkv
