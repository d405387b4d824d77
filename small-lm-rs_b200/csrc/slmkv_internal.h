// Definitions shared by the host engine (slmkv_host.cpp) and the kernels
// (slmkv_kernels.cu). Plain structs only: they are copied to the device as
// kernel parameters or as the uploaded step descriptor.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "slmkv.h"
#include "slmkv_timeline.h"

namespace slmkv {

constexpr int kBlockTokens = 16;  // tokens per physical block
constexpr int kHeadDim = 64;      // the head width the kernels are built for

// Per-sequence entry of an uploaded step descriptor.
struct SeqEntry {
  int32_t slot;        // block-table row
  int32_t base;        // position of the first new token (pre-append length)
  int32_t count;       // new tokens this step
  int32_t row_offset;  // first row of this sequence in the batch's token rows
  int32_t ctx_len;     // tokens attended by the last new token (base + count)
  int32_t pad[3];
};

// Decode plan, one entry per (sequence, KV head) in batch order. The step's
// blocks form one stream of chunk ids (chunk = physical block * Hkv + head),
// pair after pair; `blk_begin` is where this pair's blocks start in it.
struct PairEntry {
  int32_t seq;         // batch row of q / out / new K,V / status
  int32_t head;        // KV head
  int32_t ctx_len;     // tokens attended (the new token sits at ctx_len-1 when fused)
  int32_t blk_begin;   // first stream index of this pair
  int32_t nblk;        // stream entries of this pair (= ceil(ctx_len / 16))
  int32_t part_base;   // first split-K partial slot (when nseg > 1)
  int32_t first_warp;  // decode warp that owns stream index blk_begin
  int32_t nseg;        // decode warps covering this pair; bit 30 set when the
                       // pair starts exactly where its first warp's range starts
};
static_assert(sizeof(PairEntry) == 32, "PairEntry is read as two int4");

// Decode CTA shape (one CTA per SM): warps per CTA and K/V stages per warp,
// per pool type and query heads per KV head, sized to the 227 KiB of shared
// memory (each stage holds one 16-token block of K and V plus side inputs).
// Twelve warps per SM hide the per-block latency best where they fit in
// shared memory (measured on the batched decode microbench for f32 with at
// most two query heads per KV head, 12 x 1 against 10 x 2 and 16 x 1, and
// again with a step's 8 layers in one launch: 12 x 1 against 10 x 2, 11 x 2
// and 8 x 2; and on
// the scaled GQA shape for bf16 with four, 12 x 2 against 8 x 4, 8 x 2 and
// 16 x 1). Larger query groups need more shared memory per warp.
constexpr int decode_warps(int bf16, int group) {
  return (bf16 ? group <= 4 : group <= 2) ? 12 : 8;
}
constexpr int decode_stages(int bf16, int group) {
  return bf16 ? (group <= 4 ? 2 : 3) : (group <= 2 ? 1 : 2);
}
constexpr int kMaxDecodeWarps = 12;  // the largest decode_warps()
static_assert(decode_warps(0, 1) <= kMaxDecodeWarps && decode_warps(0, 8) <= kMaxDecodeWarps &&
                  decode_warps(1, 1) <= kMaxDecodeWarps && decode_warps(1, 8) <= kMaxDecodeWarps,
              "kMaxDecodeWarps bounds every decode CTA shape");

// Block-table write or copy-on-write job, applied before a step's kernels.
struct TableUpdate {
  int32_t slot, index, block, pad;
};
struct CopyJob {
  int32_t src, dst;
};

// Device status words (per batch sequence, and one per context).
// kStatusNonFinite: appended K/V not finite (kv_cache.rs:192-197);
// kStatusNonFiniteScore: an attention score not finite (softmax.rs:17-22).
enum : int32_t { kStatusNonFinite = 1, kStatusNonFiniteScore = 2 };
// Device error word bits: a bounded wait expired; a block table held an id
// outside the pool; a kernel found its shared-memory layout misaligned.
enum : int32_t { kErrTimeout = 1, kErrBadBlock = 2, kErrLayout = 4, kErrBadToken = 8, kErrLogits = 16 };

struct PoolGeom {
  void* k;                   // pool base (layer 0)
  void* v;
  int64_t layer_elems;       // elements per layer per pool
  int32_t* block_table;      // [max_sequences][max_blocks_per_seq]
  int32_t max_blocks_per_seq;
  int32_t num_blocks;
  int32_t num_layers;
  int32_t kv_heads;
  int32_t q_heads;
  int32_t bf16;              // element type of the pools
  const float2* rope;        // [context_length][head_dim/2] (cos, sin)
  int32_t context_length;
  int32_t* error;            // context error word (kErr* bits)
};


// ---- kernel launchers (slmkv_kernels.cu) ----------------------------------
// Layers one decode launch may run (consecutive layers, one plan; f32
// pools: on the scaled GQA shape a bf16 launch of several layers measured
// slower than one launch per layer, 36.7 against 34.4 us a layer).
constexpr int kMaxLaunchLayers = 8;

struct StreamDecodeLaunch {
  PoolGeom g;
  int32_t layer;     // first layer of the launch
  int32_t n_layers;  // layers layer .. layer + n_layers - 1, 1..kMaxLaunchLayers
  const PairEntry* pairs;
  int32_t n_pairs;
  const int32_t* chunks;          // [total_blocks]
  int32_t total_blocks;
  const int4* warp_start;         // [2 * n_warps]: {first pair, seq, head,
                                  //  ctx_len}, {first pair's end, g0, g1, 0}
  int32_t n_warps;                // grid = ceil(n_warps / decode_warps()) CTAs
  // per layer of the launch:
  const float* q[kMaxLaunchLayers];      // [n, Hq, d]
  const float* k_new[kMaxLaunchLayers];  // [n, Hkv, d] (fused mode) or null
  const float* v_new[kMaxLaunchLayers];
  float* out[kMaxLaunchLayers];          // [n, Hq, d]
  uint32_t* out_bf16;  // one-layer launches: out rounded to bf16 as well (or null)
  float* part_acc;        // [layer of the launch][part_stride slots][G][d]
  float2* part_ml;        // [layer][part_stride][G] (running max in the exp2 domain, sum)
  int32_t part_stride;    // split-K partial slots per layer of the launch
  int32_t* counters;      // [layer][counter_stride], zero between launches
  int32_t counter_stride;
  int32_t* status;     // [n]
  int32_t fused;       // 1: rope(q,k) + append + attend; 0: attend (q rotated)
  // 1: this layer's pool region was last written by a launch that completed
  // before the previous kernel of the stream started, so the first K/V stages
  // may be fetched before waiting on that kernel (set by the host).
  int32_t early_kv;
  // bf16 pools: TMA maps of the whole K and V pools as rows of 64 bf16
  // (row = ((layer * num_blocks + block) * kv_heads + head) * 16 + slot), box
  // 16 rows, 128-byte swizzle. Unused for f32 pools.
  CUtensorMap tmap_k, tmap_v;
};
cudaError_t launch_decode(const StreamDecodeLaunch& p, cudaStream_t s);

struct AppendLaunch {
  PoolGeom g;
  int32_t layer;
  const SeqEntry* seqs;
  int32_t n_seq;
  int32_t total_tokens;
  const float* k_in;   // [total_tokens, Hkv, d]
  const float* v_in;
  int32_t rotate;
  int32_t* status;     // [n_seq]
};
cudaError_t launch_append(const AppendLaunch& p, cudaStream_t s);

struct GatherLaunch {
  PoolGeom g;
  int32_t layer;
  int32_t slot;
  int32_t length;
  float* k_out;  // [length, Hkv, d] or null
  float* v_out;
};
cudaError_t launch_gather(const GatherLaunch& p, cudaStream_t s);

struct PrefillLaunch {
  PoolGeom g;
  int32_t layer;
  const SeqEntry* seqs;
  int32_t n_seq;
  int32_t total_tokens;
  const float* q;  // [total_tokens, Hq, d]
  int32_t rotate;
  float* out;
  int32_t max_count;  // largest per-sequence token count
  int32_t* status;    // [n_seq]: kStatusNonFiniteScore when a score is not finite
  int32_t max_ctx;    // exact-order attention: the longest row (positions attended)
  // exact-order decode (token counts 1): the new K (unrotated) and V rows
  // [n, kv_heads, d], appended by the attention kernel itself
  const float* k_new;
  const float* v_new;
  int32_t fused;
  CUtensorMap tmap_k, tmap_v;  // bf16 pools: the decode kernel's pool maps
};
cudaError_t launch_prefill(const PrefillLaunch& p, cudaStream_t s);
// Attention in the reference's operation order, bit for bit (f32 pools);
// its shared memory per launch, and the longest row a launch can take.
cudaError_t launch_exact_attention(const PrefillLaunch& p, cudaStream_t s);
constexpr int32_t kExactMaxCtx = 48 * 1024;
// bf16 pools on the tensor cores (tcgen05): slmkv_prefill_tc.cu.
bool prefill_tc_supported(const PrefillLaunch& p);
cudaError_t launch_prefill_tc(const PrefillLaunch& p, cudaStream_t s);

cudaError_t launch_apply_updates(const PoolGeom& g, const TableUpdate* updates, int32_t n_updates,
                                 const CopyJob* copies, int32_t n_copies, cudaStream_t s);

// ---- few-row projections on the tensor cores (slmkv_rowgemm.cu) ----
enum : int { kRowQKV = 0, kRowO = 1, kRowGU = 2, kRowDown = 3, kRowHead = 4 };
struct RowGemmLaunch {
  CUtensorMap tmap_w;  // weights [K][ld] bf16, 64 x 64 boxes, 128-byte swizzle
  CUtensorMap tmap_x;  // rows [rows][K] bf16 (encoded by launch_row_gemm)
  const void* x;
  int32_t rows, K;
  int32_t ncols;  // output columns (QKV: H + 2 KV; O, Down: H; GU: I)
  int32_t H, KV, I;
  int32_t nchunks, chunks_per_split;  // filled by launch_row_gemm
  float* y0;     // QKV: q; O, Down: the residual stream (accumulated)
  float* y1;     // QKV: k
  float* y2;     // QKV: v
  void* h;       // GU: [rows][I] bf16
  float beta_gate, beta_up;
  int32_t* err;
  // The RMSNorm in front of q/k/v and gate/up, applied across the GEMM:
  // O and Down with norm_next set also write the next projection's operand
  // bf16(x * norm_next) into xg [rows][H] and each row's sum of squares over
  // their 128-column tile into ssq [rows][ssq_ld]; QKV and GU with ssq_in set
  // scale each row's reduced sums by 1 / sqrt(sum over the tiles / H + eps).
  const float* norm_next;
  void* xg;
  float* ssq;
  const float* ssq_in;
  int32_t ssq_ld;
  float eps;
};
struct RowGemmPlan {
  int32_t rt, row_tiles, col_tiles, nchunks, chunks_per_split, splits;
};
RowGemmPlan plan_row_gemm(int mode, int32_t rows, int32_t K, int32_t ncols, int32_t sms);
cudaError_t encode_row_gemm_map(CUtensorMap* map, const void* base, int32_t inner, int32_t outer,
                                int32_t box_inner, int32_t box_outer);
cudaError_t launch_row_gemm(int mode, RowGemmLaunch p, const RowGemmPlan& q, cudaStream_t s);

// ---- the model step's view of a context and an open batch (slmkv_host.cpp) ----
struct BatchRows {
  cudaStream_t stream;
  int32_t n_seq;
  int32_t total_tokens;
  const int32_t* counts;  // [n_seq], host
  const SeqEntry* d_seqs; // [n_seq], device: row_offset, count, base per sequence
};
BatchRows batch_rows(const slm_batch* b);
// slm_batch_decode_layer that also writes its output rounded to bf16
// (d_out_bf16: [n, q_heads * d / 2] bf16 pairs), for the next projection.
slm_status batch_decode_layer_bf16(slm_batch* b, int32_t layer, const float* d_query,
                                   const float* d_keys, const float* d_values, float* d_out,
                                   uint32_t* d_out_bf16);
slm_ctx* batch_ctx(const slm_batch* b);
int32_t* ctx_error_word(slm_ctx* c);
void ctx_count_launches(slm_ctx* c, int32_t n);
// Selects the context's device; SLM_ERR_NO_DEVICE for a host-only context.
slm_status ctx_need_device(slm_ctx* c);
// Sets the context's last error message and returns code.
slm_status ctx_fail(slm_ctx* c, slm_status code, const char* msg);

}  // namespace slmkv
