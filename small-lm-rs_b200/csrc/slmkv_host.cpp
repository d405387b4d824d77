// Host engine of the KV-cache hot path: paged block pool, per-sequence
// per-layer lengths (the reference's KvCache bookkeeping, kv_cache.rs:89-412),
// prefix index, step descriptors, and the C ABI declared in include/slmkv.h.
//
// Error messages follow EngineError's Display format (error.rs:14-60):
//   "invalid model configuration: <message>"
//   "invalid input for <component>: <message>"
#include <algorithm>
#include <array>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <new>
#include <random>
#include <string>
#include <deque>
#include <unordered_map>
#include <vector>

#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "slmkv.h"
#include "slmkv_internal.h"

using namespace slmkv;

namespace {

// Batches that may be submitted and not yet resolved at once (the host may
// plan and queue that many steps ahead of the GPU, so that a stall of the
// host thread of up to that many steps leaves the GPU busy), and readback
// slots (one more, for slm_batch_end while that many are in flight).
constexpr int kMaxInFlight = 8;
// Descriptor slots: every submitted batch and the open one hold their own.
constexpr int kUploadSlots = kMaxInFlight + 1;
constexpr int kReadbackSlots = kMaxInFlight + 1;

struct Seq {
  bool live = false;
  int32_t max_len = 0;
  std::vector<int32_t> layer_len;
  std::vector<int32_t> blocks;  // logical block -> physical id
  bool in_batch = false;  // in the open batch
  int32_t in_flight = 0;  // submitted batches not yet resolved that hold it
};

struct BlockMeta {
  bool indexed = false;
  int32_t parent = -1;  // physical id of the previous block of the chain
  uint64_t key = 0;
  uint64_t stamp = 0;
  std::array<uint32_t, kBlockTokens> tokens{};
};

// Pinned staging (a ring of kUploadSlots) feeding device memory. A single device region
// is written on the caller's stream; a dual one (the batch descriptors) has a
// device buffer per slot, written on the context's copy stream while the
// previous step's kernels run, once the kernels that last read that buffer
// are done (`consumed`), with the caller's stream waiting for the copy.
struct Upload {
  uint8_t* h[kUploadSlots] = {};
  cudaEvent_t ev[kUploadSlots] = {};        // copy of slot k done
  cudaEvent_t consumed[kUploadSlots] = {};  // kernels reading slot k done
  uint8_t* d = nullptr;                     // single
  uint8_t* dd[kUploadSlots] = {};           // dual
  bool dual = false;
  size_t cap = 0;
  int next = 0, last = 0;
  uint8_t* device() const { return dual ? dd[last] : d; }   // of the last upload
};

// Decode plan of one step, built on the host (which owns every block id).
struct StreamPlan {
  std::vector<PairEntry> pairs;
  std::vector<int32_t> chunks;
  // 2 per warp: {first pair, seq, head, ctx_len}, {first pair's end, g0, g1, 0}
  std::vector<int4> warp_start;
  std::vector<int32_t> bounds;  // warp boundaries in the stream (scratch)
  // A launch that runs several layers keeps each warp's chunk ids and pair
  // entries in one 32-entry window: true when every warp's slice has at most
  // 32 blocks and touches at most 32 pairs.
  bool fits_window = false;
  std::vector<int32_t> bucket_top, bucket_next, heads_left;  // pair packing (scratch)
};

// Device addresses of one uploaded step descriptor.
struct StepDev {
  SeqEntry* seqs = nullptr;
  int32_t* status = nullptr;
  PairEntry* pairs = nullptr;
  int32_t* chunks = nullptr;
  int4* wfp = nullptr;  // warp start records
};

size_t align16(size_t x) { return (x + 15) & ~static_cast<size_t>(15); }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

uint64_t mix64(uint64_t x) {  // splitmix64 finaliser
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

}  // namespace

struct slm_batch {
  slm_ctx* ctx = nullptr;
  cudaStream_t stream = nullptr;
  std::vector<int32_t> seq_ids, counts, base;
  int32_t total_tokens = 0, max_count = 0;
  int32_t n_pairs = 0, total_blocks = 0;  // decode plan (when every count is 1)
  std::vector<uint8_t> layer_done;
  StepDev dev;
  int32_t up_slot = 0;  // descriptor slot (its `consumed` event is recorded at the end)
  // Submitted (slm_batch_submit): its status readback slot; per sequence
  // whether every layer advanced, and a rollback forced by an earlier batch
  // (poison_base >= 0: roll back to at most that length with poison_code).
  bool submitted = false, resolved = false;
  int32_t rb_slot = -1;
  std::vector<uint8_t> complete;
  std::vector<int32_t> poison_base, poison_code;
  // Resolved: per-sequence status, the first failure and its message.
  std::vector<int32_t> codes;
  slm_status first = SLM_OK;
  std::string msg;
};

struct slm_ctx {
  slm_config cfg{};
  int32_t device = -1;
  int32_t num_sms = 0;
  int32_t max_blocks_per_seq = 0;
  int32_t group = 1;
  int32_t n_warps = 0;     // decode grid: SMs x decode_warps()
  int32_t max_pairs = 0;   // max_sequences x Hkv
  int32_t launch_layers = 1;  // layers one decode launch may run (split-K scratch copies)
  int64_t max_chunks = 0;  // max_sequences x blocks per sequence x Hkv
  int64_t device_bytes = 0;
  int64_t launches = 0;  // kernels launched by this context
  // Layer of the last launch when it was a batch decode, else -1: a batch
  // decode of another layer right after it may fetch its first K/V stages
  // before waiting on it (nothing else has written the pool since).
  int32_t prev_decode_layer = -1;
  int32_t prev_decode_last = -1;  // with it, the last layer that launch ran
  std::string err;
  size_t counter_bytes() const {
    return sizeof(int32_t) * static_cast<size_t>(max_pairs) * launch_layers;
  }

  // device memory
  void* k_pool = nullptr;
  void* v_pool = nullptr;
  int32_t* d_block_table = nullptr;
  float2* d_rope = nullptr;
  float* d_part_acc = nullptr;
  float2* d_part_ml = nullptr;
  int32_t* d_counters = nullptr;
  int32_t* d_error = nullptr;
  int32_t* h_readback = nullptr;  // pinned: [1 + max_sequences]
  CUtensorMap tmap_k{}, tmap_v{};  // bf16 pools: TMA maps for the decode kernel
  // Pinned status readback of submitted batches: kReadbackSlots slots of
  // [error word, pad, status x max_sequences], each with its event.
  int32_t* h_rb = nullptr;
  cudaEvent_t rb_ev[kReadbackSlots] = {};
  bool rb_busy[kReadbackSlots] = {};
  std::deque<slm_batch*> submitted;  // oldest first
  // Batch descriptors go in on copy_stream; statuses come back on
  // readback_stream (a readback waits for its step's kernels, and must not
  // hold up the next step's descriptor behind it).
  cudaStream_t copy_stream = nullptr, readback_stream = nullptr;
  Upload up_batch, up_aux;
  // slm_batch_decode_layers_host: device staging of a step's inputs and
  // outputs, one set per descriptor slot (the batch's up_slot), grown on
  // demand. Inputs go in on io_h2d (not copy_stream, so that the next step's
  // descriptor does not queue behind them), outputs come back on
  // readback_stream ahead of the step's statuses.
  struct HostIo {
    float* d_in[kUploadSlots] = {};
    float* d_out[kUploadSlots] = {};
    size_t in_cap = 0, out_cap = 0;  // floats a slot
    cudaEvent_t in_done[kUploadSlots] = {};  // the slot's inputs are on the device
    cudaEvent_t used[kUploadSlots] = {};     // the slot's kernels are done with it
    cudaEvent_t read[kUploadSlots] = {};     // the slot's outputs are on the host
    cudaStream_t h2d = nullptr;
  } io;
  size_t upd_cap = 0, copy_cap = 0;

  // host state
  std::vector<Seq> seqs;
  std::vector<int32_t> free_slots;
  std::vector<int32_t> refcount;
  std::vector<int32_t> free_list;
  std::vector<BlockMeta> meta;
  std::unordered_multimap<uint64_t, int32_t> index;
  int32_t indexed_blocks = 0;
  uint64_t clock = 0;
  std::vector<TableUpdate> pending_updates;
  std::vector<CopyJob> pending_copies;
  slm_batch* open_batch = nullptr;
  StreamPlan plan;  // decode plan of the open batch (reused storage)

  PoolGeom geom() const {
    PoolGeom g{};
    g.k = k_pool;
    g.v = v_pool;
    g.layer_elems = static_cast<int64_t>(cfg.num_blocks) * cfg.num_key_value_heads * kBlockTokens *
                    cfg.head_dimension;
    g.block_table = d_block_table;
    g.max_blocks_per_seq = max_blocks_per_seq;
    g.num_blocks = cfg.num_blocks;
    g.num_layers = cfg.num_layers;
    g.kv_heads = cfg.num_key_value_heads;
    g.q_heads = cfg.num_query_heads;
    g.bf16 = cfg.kv_dtype == SLM_KV_BF16;
    g.rope = d_rope;
    g.context_length = cfg.context_length;
    g.error = d_error;
    return g;
  }
};

namespace {

slm_status fail(slm_ctx* ctx, slm_status code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (ctx) ctx->err = buf;
  return code;
}
slm_status input_error(slm_ctx* ctx, slm_status code, const char* component, const char* fmt,
                       ...) {
  char msg[400];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof msg, fmt, ap);
  va_end(ap);
  return fail(ctx, code, "invalid input for %s: %s", component, msg);
}
slm_status cuda_fail(slm_ctx* ctx, cudaError_t e, const char* what) {
  return fail(ctx, SLM_ERR_CUDA, "CUDA error in %s: %s", what, cudaGetErrorString(e));
}
#define CU(ctx, call)                                      \
  do {                                                     \
    cudaError_t _e = (call);                               \
    if (_e != cudaSuccess) return cuda_fail(ctx, _e, #call); \
  } while (0)

bool has_device(const slm_ctx* c) { return c->device >= 0; }

slm_status need_device(slm_ctx* c) {
  if (!has_device(c))
    return fail(c, SLM_ERR_NO_DEVICE,
                "no device: this context was created for host bookkeeping only");
  cudaError_t e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return cuda_fail(c, e, "cudaSetDevice");
  return SLM_OK;
}

Seq* get_seq(slm_ctx* c, int32_t id) {
  if (id < 0 || id >= static_cast<int32_t>(c->seqs.size()) || !c->seqs[id].live) return nullptr;
  return &c->seqs[id];
}
const Seq* get_seq(const slm_ctx* c, int32_t id) {
  if (id < 0 || id >= static_cast<int32_t>(c->seqs.size()) || !c->seqs[id].live) return nullptr;
  return &c->seqs[id];
}
slm_status unknown_seq(slm_ctx* c, int32_t id) {
  return input_error(c, SLM_ERR_INVALID_INPUT, "KV cache", "sequence %d is not live", id);
}

int32_t seq_min_len(const Seq& s) { return *std::min_element(s.layer_len.begin(), s.layer_len.end()); }
int32_t seq_max_len(const Seq& s) { return *std::max_element(s.layer_len.begin(), s.layer_len.end()); }
bool seq_synchronized(const Seq& s) { return seq_min_len(s) == seq_max_len(s); }

// ---- block pool -------------------------------------------------------------

void unindex_block(slm_ctx* c, int32_t b) {
  BlockMeta& m = c->meta[b];
  if (!m.indexed) return;
  auto range = c->index.equal_range(m.key);
  for (auto it = range.first; it != range.second; ++it)
    if (it->second == b) {
      c->index.erase(it);
      break;
    }
  m.indexed = false;
  --c->indexed_blocks;
}

void release_block(slm_ctx* c, int32_t b) {
  if (--c->refcount[b] == 0) c->free_list.push_back(b);
}

// Takes a free block, evicting the least recently used block that only the
// prefix index still holds when the free list is empty. -1 if none.
int32_t take_block(slm_ctx* c) {
  if (c->free_list.empty()) {
    int32_t victim = -1;
    uint64_t best = UINT64_MAX;
    for (int32_t b = 0; b < c->cfg.num_blocks; ++b)
      if (c->meta[b].indexed && c->refcount[b] == 1 && c->meta[b].stamp < best) {
        best = c->meta[b].stamp;
        victim = b;
      }
    if (victim < 0) return -1;
    unindex_block(c, victim);
    release_block(c, victim);
  }
  const int32_t b = c->free_list.back();
  c->free_list.pop_back();
  c->refcount[b] = 1;
  return b;
}

void release_tail(slm_ctx* c, int32_t slot, int32_t keep_blocks) {
  Seq& s = c->seqs[slot];
  while (static_cast<int32_t>(s.blocks.size()) > keep_blocks) {
    release_block(c, s.blocks.back());
    s.blocks.pop_back();
  }
}

int32_t blocks_for(int32_t tokens) { return (tokens + kBlockTokens - 1) / kBlockTokens; }

// Ensures seq has exclusive blocks covering positions [from, to). New blocks
// and copy-on-write replacements are recorded in `taken` (for undo) and the
// pending table updates / copies. Returns false when the pool is exhausted.
struct Undo {
  std::vector<std::pair<int32_t, std::vector<int32_t>>> old_blocks;  // slot, previous block list
  std::vector<int32_t> taken;
  size_t updates_mark = 0, copies_mark = 0;
};

bool reserve_positions(slm_ctx* c, int32_t slot, int32_t from, int32_t to, Undo& undo) {
  Seq& s = c->seqs[slot];
  if (to <= from) return true;
  const int32_t first = from / kBlockTokens, last = (to - 1) / kBlockTokens;
  bool saved = false;
  auto save = [&] {
    if (!saved) {
      undo.old_blocks.emplace_back(slot, s.blocks);
      saved = true;
    }
  };
  for (int32_t j = first; j <= last; ++j) {
    if (j < static_cast<int32_t>(s.blocks.size())) {
      const int32_t b = s.blocks[j];
      if (c->refcount[b] > 1) {  // shared: copy before writing
        const int32_t nb = take_block(c);
        if (nb < 0) return false;
        save();
        undo.taken.push_back(nb);
        c->pending_copies.push_back(CopyJob{b, nb});
        c->pending_updates.push_back(TableUpdate{slot, j, nb, 0});
        release_block(c, b);
        s.blocks[j] = nb;
      }
    } else {
      const int32_t nb = take_block(c);
      if (nb < 0) return false;
      save();
      undo.taken.push_back(nb);
      c->pending_updates.push_back(TableUpdate{slot, j, nb, 0});
      s.blocks.push_back(nb);
    }
  }
  return true;
}

void rollback_reserve(slm_ctx* c, Undo& undo) {
  // Restore block lists (this re-acquires shared blocks released by COW).
  for (auto it = undo.old_blocks.rbegin(); it != undo.old_blocks.rend(); ++it) {
    Seq& s = c->seqs[it->first];
    for (int32_t b : it->second)
      if (std::find(s.blocks.begin(), s.blocks.end(), b) == s.blocks.end()) ++c->refcount[b];
    s.blocks = it->second;
  }
  for (int32_t b : undo.taken) {
    c->refcount[b] = 0;
    c->free_list.push_back(b);
  }
  c->pending_updates.resize(undo.updates_mark);
  c->pending_copies.resize(undo.copies_mark);
}

// ---- uploads ------------------------------------------------------------------

slm_status upload_alloc(slm_ctx* c, Upload& u, size_t cap, bool dual) {
  u.cap = cap;
  u.dual = dual;
  for (int k = 0; k < kUploadSlots; ++k) {
    CU(c, cudaMallocHost(reinterpret_cast<void**>(&u.h[k]), cap));
    CU(c, cudaEventCreateWithFlags(&u.ev[k], cudaEventDisableTiming));
    CU(c, cudaEventCreateWithFlags(&u.consumed[k], cudaEventDisableTiming));
    if (dual) {
      CU(c, cudaMalloc(reinterpret_cast<void**>(&u.dd[k]), cap));
      c->device_bytes += static_cast<int64_t>(cap);
    }
  }
  if (!dual) {
    CU(c, cudaMalloc(reinterpret_cast<void**>(&u.d), cap));
    c->device_bytes += static_cast<int64_t>(cap);
  }
  return SLM_OK;
}
void upload_free(Upload& u) {
  for (int k = 0; k < kUploadSlots; ++k) {
    if (u.h[k]) cudaFreeHost(u.h[k]);
    if (u.ev[k]) cudaEventDestroy(u.ev[k]);
    if (u.consumed[k]) cudaEventDestroy(u.consumed[k]);
    if (u.dd[k]) cudaFree(u.dd[k]);
    u.h[k] = u.dd[k] = nullptr;
    u.ev[k] = u.consumed[k] = nullptr;
  }
  if (u.d) cudaFree(u.d);
  u.d = nullptr;
}
uint8_t* upload_begin(Upload& u) {
  cudaEventSynchronize(u.ev[u.next]);
  return u.h[u.next];
}
cudaError_t upload_end(Upload& u, size_t bytes, cudaStream_t s, cudaStream_t copy) {
  const int k = u.next;
  cudaError_t e;
  if (u.dual) {
    e = cudaStreamWaitEvent(copy, u.consumed[k], 0);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(u.dd[k], u.h[k], bytes, cudaMemcpyHostToDevice, copy);
    if (e == cudaSuccess) e = cudaEventRecord(u.ev[k], copy);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, u.ev[k], 0);
  } else {
    e = cudaMemcpyAsync(u.d, u.h[k], bytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaEventRecord(u.ev[k], s);
  }
  u.last = k;
  u.next = (k + 1) % kUploadSlots;
  return e;
}

// Layout of one upload: [seqs][status][pairs][chunks][warp start records]
// [table updates][copy jobs].
struct DescLayout {
  size_t seqs = 0, status = 0, pairs = 0, chunks = 0, wfp = 0, updates = 0, copies = 0, total = 0;
};
DescLayout desc_layout(size_t n, size_t n_pairs, size_t n_chunks, size_t n_warps, size_t nu,
                       size_t nc) {
  DescLayout L;
  L.seqs = 0;
  L.status = align16(L.seqs + sizeof(SeqEntry) * n);
  L.pairs = align16(L.status + sizeof(int32_t) * n);
  L.chunks = align16(L.pairs + sizeof(PairEntry) * n_pairs);
  L.wfp = align16(L.chunks + sizeof(int32_t) * n_chunks);
  L.updates = align16(L.wfp + 2 * sizeof(int4) * n_warps);
  L.copies = align16(L.updates + sizeof(TableUpdate) * nu);
  L.total = align16(L.copies + sizeof(CopyJob) * nc);
  return L;
}

// Sends pending table updates / copies that would not fit into a descriptor
// upload, through the aux region, and applies them.
slm_status flush_excess(slm_ctx* c, cudaStream_t s, size_t keep_updates, size_t keep_copies) {
  while (c->pending_updates.size() > keep_updates || c->pending_copies.size() > keep_copies) {
    const size_t nu = std::min(c->pending_updates.size(), c->upd_cap);
    const size_t nc = std::min(c->pending_copies.size(), c->copy_cap);
    DescLayout L = desc_layout(0, 0, 0, 0, nu, nc);
    uint8_t* h = upload_begin(c->up_aux);
    memcpy(h + L.updates, c->pending_updates.data(), nu * sizeof(TableUpdate));
    memcpy(h + L.copies, c->pending_copies.data(), nc * sizeof(CopyJob));
    CU(c, upload_end(c->up_aux, L.total, s, c->copy_stream));
    c->prev_decode_layer = -1;
    CU(c, launch_apply_updates(c->geom(), reinterpret_cast<TableUpdate*>(c->up_aux.d + L.updates),
                               static_cast<int32_t>(nu),
                               reinterpret_cast<CopyJob*>(c->up_aux.d + L.copies),
                               static_cast<int32_t>(nc), s));
    ++c->launches;
    c->pending_updates.erase(c->pending_updates.begin(), c->pending_updates.begin() + nu);
    c->pending_copies.erase(c->pending_copies.begin(), c->pending_copies.begin() + nc);
  }
  return SLM_OK;
}

// Builds the decode plan for sequences (batch rows) attending `ctx_len`
// tokens: one PairEntry per (row, KV head), the chunk stream, and an equal
// split of the stream over the decode warps: warp w owns stream indices
// [floor(w*T/NW), floor((w+1)*T/NW)); W consecutive warps form one CTA.
//
// The pairs are ordered so that they fill each CTA's share of the stream
// exactly: for the CTA being filled, the largest remaining pair that fits its
// remaining room goes next. Only when no remaining pair fits is one cut across
// the CTA boundary (the largest, so long contexts are cut and short ones are
// not). A pair inside one CTA merges its warps' partials in shared memory; a
// cut pair merges through global memory at the end of the kernel, which is
// the kernel's tail, so the ordering removes most of that tail. Warp bounds
// are stepped without divisions and matched to pairs in one sweep.
void build_stream_plan(const slm_ctx* c, const std::vector<SeqEntry>& entries, int32_t n_warps,
                       StreamPlan& plan) {
  const int32_t Hkv = c->cfg.num_key_value_heads;
  const int32_t W = decode_warps(c->cfg.kv_dtype == SLM_KV_BF16, c->group);
  const int32_t n_pairs = static_cast<int32_t>(entries.size()) * Hkv;
  int64_t T = 0;
  int32_t maxb = 0;
  for (const SeqEntry& e : entries) {
    const int32_t nb = blocks_for(e.ctx_len);
    T += static_cast<int64_t>(nb) * Hkv;
    maxb = std::max(maxb, nb);
  }
  const int32_t NW = static_cast<int32_t>(std::min<int64_t>(n_warps, T));
  // bounds[w] = floor(w*T/NW): T = q*NW + r, carry r each step.
  std::vector<int32_t>& bounds = plan.bounds;
  bounds.resize(static_cast<size_t>(NW) + 1);
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
  // Rows bucketed by block count (all heads of a row have the same count);
  // a stack per bucket, rows pushed in reverse so each pops in row order.
  std::vector<int32_t>& top = plan.bucket_top;
  std::vector<int32_t>& next = plan.bucket_next;
  top.assign(static_cast<size_t>(maxb) + 1, -1);
  next.resize(entries.size());
  for (int32_t i = static_cast<int32_t>(entries.size()) - 1; i >= 0; --i) {
    const int32_t nb = blocks_for(entries[i].ctx_len);
    next[i] = top[nb];
    top[nb] = i;
  }
  std::vector<int32_t>& heads_left = plan.heads_left;
  heads_left.assign(entries.size(), Hkv);
  int32_t hi = maxb;  // no non-empty bucket above this
  auto take = [&](int32_t nb) {  // pops one pair of a row from bucket nb
    const int32_t i = top[nb];
    const int32_t h = Hkv - heads_left[i];
    if (--heads_left[i] == 0) top[nb] = next[i];
    return std::make_pair(i, h);
  };

  plan.pairs.resize(static_cast<size_t>(n_pairs));
  plan.chunks.resize(static_cast<size_t>(T));
  int32_t pos = 0, wcta = 0;  // stream position; first warp of the CTA being filled
  for (int32_t k = 0; k < n_pairs; ++k) {
    while (wcta + W < NW && bounds[wcta + W] <= pos) wcta += W;
    const int32_t room = bounds[std::min(wcta + W, NW)] - pos;
    while (hi > 0 && top[hi] < 0) --hi;
    int32_t nb = std::min(room, hi);
    while (nb > 0 && top[nb] < 0) --nb;
    if (nb <= 0) nb = hi;  // nothing fits: cut the largest across the boundary
    const auto [i, h] = take(nb);
    const SeqEntry& e = entries[i];
    PairEntry& pe = plan.pairs[k];
    pe = PairEntry{};
    pe.seq = i;
    pe.head = h;
    pe.ctx_len = e.ctx_len;
    pe.blk_begin = pos;
    pe.nblk = nb;
    const int32_t* blocks = c->seqs[e.slot].blocks.data();
    int32_t* out = plan.chunks.data() + pos;
    for (int32_t j = 0; j < nb; ++j) out[j] = blocks[j] * Hkv + h;
    pos += nb;
  }
  // Owner of stream index x: the w with bounds[w] <= x < bounds[w+1]; the
  // queries below only move forward, so a cursor per query suffices.
  int32_t wa = 0, wb = 0, part = 0;
  for (PairEntry& pe : plan.pairs) {
    while (bounds[wa + 1] <= pe.blk_begin) ++wa;
    const int32_t last = pe.blk_begin + pe.nblk - 1;
    if (wb < wa) wb = wa;
    while (bounds[wb + 1] <= last) ++wb;
    pe.first_warp = wa;
    pe.nseg = wb - wa + 1;
    if (bounds[wa] == pe.blk_begin) pe.nseg |= (1 << 30);
    pe.part_base = part;
    // Pairs merge per CTA first (W consecutive warps); a pair that spans
    // CTAs gets one global partial slot per CTA it touches.
    const int32_t n_cta = wb / W - wa / W + 1;
    if (n_cta > 1) part += n_cta;
  }
  plan.warp_start.resize(static_cast<size_t>(2 * NW));
  plan.fits_window = true;
  size_t pc = 0, pl = 0;  // first and last pair of warp w's slice
  for (int32_t w = 0; w < NW; ++w) {
    const int32_t b = bounds[w];
    while (plan.pairs[pc].blk_begin + plan.pairs[pc].nblk <= b) ++pc;
    const PairEntry& pe = plan.pairs[pc];
    plan.warp_start[2 * w] = make_int4(static_cast<int32_t>(pc), pe.seq, pe.head, pe.ctx_len);
    plan.warp_start[2 * w + 1] = make_int4(pe.blk_begin + pe.nblk, b, bounds[w + 1], 0);
    if (pl < pc) pl = pc;
    while (plan.pairs[pl].blk_begin + plan.pairs[pl].nblk < bounds[w + 1]) ++pl;
    if (bounds[w + 1] - b > 32 || pl - pc + 1 > 32) plan.fits_window = false;
  }
}

// Uploads [entries, zeroed status, decode plan (optional), pending table
// updates / copies] into region `u` with one copy, and applies the updates.
slm_status upload_step(slm_ctx* c, Upload& u, cudaStream_t s, const std::vector<SeqEntry>& entries,
                       const StreamPlan* plan, StepDev* dev, bool with_table_updates = true) {
  slm_status rc = flush_excess(c, s, c->upd_cap, c->copy_cap);
  if (rc) return rc;
  const size_t n = entries.size();
  const size_t np = plan ? plan->pairs.size() : 0, nch = plan ? plan->chunks.size() : 0;
  const size_t nw = plan ? plan->warp_start.size() / 2 : 0;
  const size_t nu = with_table_updates ? c->pending_updates.size() : 0;
  const size_t nc = c->pending_copies.size();
  DescLayout L = desc_layout(n, np, nch, nw, nu, nc);
  if (L.total > u.cap)
    return fail(c, SLM_ERR_INVALID_INPUT, "invalid input for KV cache: step descriptor too large");
  uint8_t* h = upload_begin(u);
  memcpy(h + L.seqs, entries.data(), sizeof(SeqEntry) * n);
  memset(h + L.status, 0, sizeof(int32_t) * n);
  if (np) memcpy(h + L.pairs, plan->pairs.data(), sizeof(PairEntry) * np);
  if (nch) memcpy(h + L.chunks, plan->chunks.data(), sizeof(int32_t) * nch);
  if (nw) memcpy(h + L.wfp, plan->warp_start.data(), sizeof(int4) * 2 * nw);
  if (nu) memcpy(h + L.updates, c->pending_updates.data(), nu * sizeof(TableUpdate));
  if (nc) memcpy(h + L.copies, c->pending_copies.data(), nc * sizeof(CopyJob));
  CU(c, upload_end(u, L.total, s, c->copy_stream));
  uint8_t* d = u.device();
  if (nu || nc) {
    c->prev_decode_layer = -1;
    CU(c, launch_apply_updates(c->geom(), reinterpret_cast<TableUpdate*>(d + L.updates),
                               static_cast<int32_t>(nu), reinterpret_cast<CopyJob*>(d + L.copies),
                               static_cast<int32_t>(nc), s));
    ++c->launches;
    if (with_table_updates) c->pending_updates.clear();
    c->pending_copies.clear();
  }
  dev->seqs = reinterpret_cast<SeqEntry*>(d + L.seqs);
  dev->status = reinterpret_cast<int32_t*>(d + L.status);
  dev->pairs = reinterpret_cast<PairEntry*>(d + L.pairs);
  dev->chunks = reinterpret_cast<int32_t*>(d + L.chunks);
  dev->wfp = reinterpret_cast<int4*>(d + L.wfp);
  return SLM_OK;
}

// TMA maps of a bf16 pool for the decode kernel: the whole pool as rows of
// 64 bf16 (128 B; row = ((layer * num_blocks + block) * kv_heads + head) * 16
// + slot), a box of one 16-row chunk, 128-byte swizzle. The encoder comes
// from the driver through the runtime (no link against the driver library).
slm_status make_pool_maps(slm_ctx* c) {
  static const PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }();
  if (!encode) return fail(c, SLM_ERR_CUDA, "CUDA error: cuTensorMapEncodeTiled is unavailable");
  const slm_config& k = c->cfg;
  const uint64_t rows = static_cast<uint64_t>(k.num_layers) * k.num_blocks *
                        k.num_key_value_heads * kBlockTokens;
  if (rows > static_cast<uint64_t>(INT32_MAX))
    return fail(c, SLM_ERR_INVALID_CONFIGURATION,
                "invalid configuration: a bf16 pool of %llu rows exceeds the 2^31 rows a TMA "
                "coordinate addresses",
                static_cast<unsigned long long>(rows));
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k.head_dimension), rows};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k.head_dimension) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(k.head_dimension), kBlockTokens};
  const cuuint32_t estride[2] = {1, 1};
  void* pools[2] = {c->k_pool, c->v_pool};
  CUtensorMap* maps[2] = {&c->tmap_k, &c->tmap_v};
  for (int i = 0; i < 2; ++i) {
    const CUresult r = encode(maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, pools[i], dims,
                              strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(c, SLM_ERR_CUDA, "CUDA error: cuTensorMapEncodeTiled failed (%d)",
                  static_cast<int>(r));
  }
  return SLM_OK;
}

// Fills a decode launch for an uploaded plan.
StreamDecodeLaunch decode_launch(slm_ctx* c, int32_t layer, const StepDev& dev,
                                 const StreamPlan& plan) {
  StreamDecodeLaunch p{};
  p.g = c->geom();
  p.layer = layer;
  p.tmap_k = c->tmap_k;
  p.tmap_v = c->tmap_v;
  p.pairs = dev.pairs;
  p.n_pairs = static_cast<int32_t>(plan.pairs.size());
  p.chunks = dev.chunks;
  p.total_blocks = static_cast<int32_t>(plan.chunks.size());
  p.warp_start = dev.wfp;
  p.n_warps = static_cast<int32_t>(plan.warp_start.size() / 2);
  p.n_layers = 1;
  p.part_acc = c->d_part_acc;
  p.part_ml = c->d_part_ml;
  p.part_stride = c->max_pairs + c->n_warps;
  p.counters = c->d_counters;
  p.counter_stride = c->max_pairs;
  p.status = dev.status;
  return p;
}

// Reads back and clears the context error word (stream must be idle).
slm_status check_device_error(slm_ctx* c) {
  int32_t e = 0;
  CU(c, cudaMemcpy(&e, c->d_error, sizeof e, cudaMemcpyDeviceToHost));
  if (e) {
    CU(c, cudaMemset(c->d_error, 0, sizeof(int32_t)));
    CU(c, cudaMemset(c->d_counters, 0, c->counter_bytes()));
    if (e & kErrTimeout)
      return fail(c, SLM_ERR_DEVICE_TIMEOUT, "device wait timed out (error word 0x%x)", e);
    if (e & kErrLayout)
      return fail(c, SLM_ERR_CUDA, "CUDA error: a kernel found its shared memory misaligned (0x%x)", e);
    if (e & kErrBadToken)
      return fail(c, SLM_ERR_INVALID_INPUT,
                  "invalid input for embedding lookup: token id outside the vocabulary (0x%x)", e);
    if (e & kErrLogits)
      return fail(c, SLM_ERR_INVALID_INPUT,
                  "invalid input for greedy decoding: final-position logits are not finite (0x%x)", e);
    return fail(c, SLM_ERR_INVALID_INPUT,
                "invalid input for KV cache: block table held an out-of-pool id (0x%x)", e);
  }
  return SLM_OK;
}

void compute_rope_table(const slm_config& cfg, std::vector<float2>& out) {
  // rope.rs:33-36 inverse frequencies, rope.rs:90-93 angle = pos * inv and
  // sin_cos, evaluated with the same libm calls the reference lowers to.
  const int half = cfg.head_dimension / 2;
  std::vector<float> inv(half);
  const float denominator = static_cast<float>(cfg.head_dimension);
  for (int i = 0; i < half; ++i) {
    const float exponent = -(2.0f * static_cast<float>(i)) / denominator;
    inv[i] = powf(cfg.rope_theta, exponent);
  }
  out.resize(static_cast<size_t>(cfg.context_length) * half);
  for (int32_t p = 0; p < cfg.context_length; ++p) {
    const float pos = static_cast<float>(p);
    for (int i = 0; i < half; ++i) {
      const float angle = pos * inv[i];
      out[static_cast<size_t>(p) * half + i] = make_float2(cosf(angle), sinf(angle));
    }
  }
}

void destroy_device(slm_ctx* c) {
  if (!has_device(c)) return;
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  void* ptrs[] = {c->k_pool, c->v_pool, c->d_block_table, c->d_rope, c->d_part_acc,
                  c->d_part_ml, c->d_counters, c->d_error};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  if (c->h_readback) cudaFreeHost(c->h_readback);
  if (c->h_rb) cudaFreeHost(c->h_rb);
  for (cudaEvent_t ev : c->rb_ev)
    if (ev) cudaEventDestroy(ev);
  upload_free(c->up_batch);
  upload_free(c->up_aux);
  for (int k = 0; k < kUploadSlots; ++k) {
    if (c->io.d_in[k]) cudaFree(c->io.d_in[k]);
    if (c->io.d_out[k]) cudaFree(c->io.d_out[k]);
    for (cudaEvent_t ev : {c->io.in_done[k], c->io.used[k], c->io.read[k]})
      if (ev) cudaEventDestroy(ev);
  }
  if (c->io.h2d) cudaStreamDestroy(c->io.h2d);
  if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
  if (c->readback_stream) cudaStreamDestroy(c->readback_stream);
}

template <typename T>
slm_status dev_alloc(slm_ctx* c, T** p, size_t bytes, const char* what) {
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), bytes);
  if (e != cudaSuccess) return cuda_fail(c, e, what);
  c->device_bytes += static_cast<int64_t>(bytes);
  return SLM_OK;
}

slm_status finish_single(slm_ctx* c, cudaStream_t s, int32_t* d_status, int32_t* status) {
  CU(c, cudaMemcpyAsync(c->h_readback, d_status, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  CU(c, cudaStreamSynchronize(s));
  *status = c->h_readback[0];
  return check_device_error(c);
}

// Message of the last failed call on this thread that had no context
// (slm_create, slm_decode_attention_noalloc).
thread_local std::string g_create_error;

// kv_cache.rs:43-55, rope.rs:21-31 and the config.rs head-divisibility rule,
// plus the shapes the kernels are built for. Empty string = valid.
std::string validate_config(const slm_config& k) {
  if (k.num_layers <= 0 || k.num_key_value_heads <= 0 || k.head_dimension <= 0 ||
      k.num_query_heads <= 0 || k.context_length <= 0)
    return "all KV-cache dimensions must be greater than zero";
  if (k.num_query_heads % k.num_key_value_heads)
    return "num_query_heads must be divisible by num_key_value_heads";
  if (k.head_dimension % 2) return "RoPE head_dimension must be positive and even";
  if (!std::isfinite(k.rope_theta) || k.rope_theta <= 0.0f)
    return "RoPE theta must be finite and greater than zero";
  if (k.head_dimension != kHeadDim)
    return "head_dimension 64 is the only width the kernels are built for";
  const int32_t G = k.num_query_heads / k.num_key_value_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return "query heads per KV head must be 1, 2, 4 or 8";
  if (k.num_blocks <= 0 || k.max_sequences <= 0)
    return "num_blocks and max_sequences must be greater than zero";
  if (k.kv_dtype != SLM_KV_F32 && k.kv_dtype != SLM_KV_BF16)
    return "kv_dtype must be SLM_KV_F32 or SLM_KV_BF16";
  return std::string();
}

}  // namespace

namespace slmkv {
// Records the message of a failed call made without a context; read back by
// slm_last_error(NULL).
void set_contextless_error(const std::string& message) { g_create_error = message; }

BatchRows batch_rows(const slm_batch* b) {
  return BatchRows{b->stream, static_cast<int32_t>(b->seq_ids.size()), b->total_tokens,
                   b->counts.data(), b->dev.seqs};
}
slm_ctx* batch_ctx(const slm_batch* b) { return b->ctx; }
int32_t* ctx_error_word(slm_ctx* c) { return c->d_error; }
void ctx_count_launches(slm_ctx* c, int32_t n) { c->launches += n; }
slm_status ctx_need_device(slm_ctx* c) { return need_device(c); }
slm_status ctx_fail(slm_ctx* c, slm_status code, const char* msg) { return fail(c, code, "%s", msg); }
}  // namespace slmkv

// =============================================================================
// C ABI
// =============================================================================
#ifdef SLMKV_TIMELINE
// Profiling builds only (not in the public header): points every instrumented
// kernel at a device buffer of `cap` TimelineRec records and a device counter
// (null buffer: off).
extern "C" int slmkv_timeline_set(void* d_buf, void* d_count, uint32_t cap) {
  auto* b = static_cast<slmkv::TimelineRec*>(d_buf);
  auto* n = static_cast<unsigned*>(d_count);
  cudaError_t e = slmkv::timeline_set_kernels(b, n, cap);
  if (e == cudaSuccess) e = slmkv::timeline_set_model(b, n, cap);
  if (e == cudaSuccess) e = slmkv::timeline_set_rowgemm(b, n, cap);
  if (e == cudaSuccess) e = slmkv::timeline_set_prefill_tc(b, n, cap);
  return static_cast<int>(e);
}
#endif

extern "C" {

slm_status slm_create(const slm_config* config, int32_t device, slm_ctx** out) {
  if (!out || !config) return SLM_ERR_INVALID_INPUT;
  *out = nullptr;
  std::unique_ptr<slm_ctx> c(new (std::nothrow) slm_ctx());
  if (!c) return SLM_ERR_INVALID_CONFIGURATION;
  const slm_config& k = *config;
  c->cfg = k;
  std::string why = validate_config(k);
  if (!why.empty()) {
    g_create_error = "invalid model configuration: " + why;
    return SLM_ERR_INVALID_CONFIGURATION;
  }
  const int32_t G = k.num_query_heads / k.num_key_value_heads;
  c->group = G;
  c->max_blocks_per_seq = blocks_for(k.context_length);
  c->max_pairs = k.max_sequences * k.num_key_value_heads;
  c->launch_layers = std::min(k.num_layers, kMaxLaunchLayers);
  c->max_chunks = static_cast<int64_t>(c->max_pairs) * c->max_blocks_per_seq;
  c->seqs.resize(k.max_sequences);
  for (int32_t i = k.max_sequences - 1; i >= 0; --i) c->free_slots.push_back(i);
  c->refcount.assign(k.num_blocks, 0);
  c->meta.resize(k.num_blocks);
  for (int32_t b = k.num_blocks - 1; b >= 0; --b) c->free_list.push_back(b);
  c->upd_cap = std::max<size_t>(4096, 2 * static_cast<size_t>(k.max_sequences));
  c->copy_cap = std::max<size_t>(1024, static_cast<size_t>(k.max_sequences));
  c->device = device;

  if (device >= 0) {
    slm_ctx* cp = c.get();
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
      g_create_error = std::string("CUDA error in cudaSetDevice: ") + cudaGetErrorString(e);
      return SLM_ERR_CUDA;
    }
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    cp->num_sms = sms;
    cp->n_warps = sms * decode_warps(k.kv_dtype == SLM_KV_BF16, G);
    const size_t esz = k.kv_dtype == SLM_KV_BF16 ? 2 : 4;
    const size_t pool_bytes = static_cast<size_t>(k.num_layers) * k.num_blocks *
                              k.num_key_value_heads * kBlockTokens * k.head_dimension * esz;
    slm_status rc = SLM_OK;
    auto step = [&](slm_status r) {
      if (rc == SLM_OK) rc = r;
    };
    step(dev_alloc(cp, &cp->k_pool, pool_bytes, "K pool"));
    step(dev_alloc(cp, &cp->v_pool, pool_bytes, "V pool"));
    if (rc == SLM_OK && k.kv_dtype == SLM_KV_BF16) step(make_pool_maps(cp));
    const size_t bt_bytes = sizeof(int32_t) * k.max_sequences * cp->max_blocks_per_seq;
    step(dev_alloc(cp, &cp->d_block_table, bt_bytes, "block table"));
    std::vector<float2> rope;
    compute_rope_table(k, rope);
    step(dev_alloc(cp, &cp->d_rope, rope.size() * sizeof(float2), "RoPE table"));
    // A pair split over s warps takes s partial slots; at most one extra
    // slot per warp boundary: pairs + warps bounds the total.
    // One copy of the partials and counters per layer a launch may run.
    const size_t parts =
        (static_cast<size_t>(cp->max_pairs) + cp->n_warps) * G * cp->launch_layers;
    step(dev_alloc(cp, &cp->d_part_acc, parts * kHeadDim * sizeof(float), "split-K partials"));
    step(dev_alloc(cp, &cp->d_part_ml, parts * sizeof(float2), "split-K partials"));
    step(dev_alloc(cp, &cp->d_counters, cp->counter_bytes(), "split-K counters"));
    step(dev_alloc(cp, &cp->d_error, sizeof(int32_t), "error word"));
    if (rc == SLM_OK) {
      e = cudaMallocHost(reinterpret_cast<void**>(&cp->h_readback),
                         sizeof(int32_t) * (k.max_sequences + 1));
      if (e == cudaSuccess)
        e = cudaMallocHost(reinterpret_cast<void**>(&cp->h_rb),
                           sizeof(int32_t) * kReadbackSlots * (k.max_sequences + 2));
      for (int i = 0; e == cudaSuccess && i < kReadbackSlots; ++i)
        e = cudaEventCreateWithFlags(&cp->rb_ev[i], cudaEventDisableTiming);
      if (e != cudaSuccess) rc = cuda_fail(cp, e, "cudaMallocHost");
    }
    if (rc == SLM_OK) {
      const size_t batch_cap = desc_layout(k.max_sequences, cp->max_pairs, cp->max_chunks,
                                           cp->n_warps, cp->upd_cap, cp->copy_cap).total + 256;
      const size_t aux_cap =
          desc_layout(1, k.num_key_value_heads,
                      static_cast<size_t>(k.num_key_value_heads) * cp->max_blocks_per_seq,
                      cp->n_warps, cp->upd_cap, cp->copy_cap).total + 256;
      e = cudaStreamCreateWithFlags(&cp->copy_stream, cudaStreamNonBlocking);
      if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&cp->readback_stream, cudaStreamNonBlocking);
      rc = (e == cudaSuccess) ? upload_alloc(cp, cp->up_batch, batch_cap, true)
                              : cuda_fail(cp, e, "cudaStreamCreate");
      if (rc == SLM_OK) rc = upload_alloc(cp, cp->up_aux, aux_cap, false);
    }
    if (rc == SLM_OK) {
      // Unused pool memory is zero: reads of not-yet-written slots are finite.
      if ((e = cudaMemset(cp->k_pool, 0, pool_bytes)) != cudaSuccess ||
          (e = cudaMemset(cp->v_pool, 0, pool_bytes)) != cudaSuccess ||
          (e = cudaMemset(cp->d_block_table, 0, bt_bytes)) != cudaSuccess ||
          (e = cudaMemset(cp->d_counters, 0, cp->counter_bytes())) != cudaSuccess ||
          (e = cudaMemset(cp->d_error, 0, sizeof(int32_t))) != cudaSuccess ||
          (e = cudaMemcpy(cp->d_rope, rope.data(), rope.size() * sizeof(float2),
                          cudaMemcpyHostToDevice)) != cudaSuccess ||
          (e = cudaDeviceSynchronize()) != cudaSuccess)
        rc = cuda_fail(cp, e, "context initialisation");
    }
    if (rc != SLM_OK) {
      g_create_error = cp->err;
      destroy_device(cp);
      return rc;
    }
  }
  g_create_error.clear();
  *out = c.release();
  return SLM_OK;
}

slm_status slm_destroy(slm_ctx* ctx) {
  if (!ctx) return SLM_ERR_INVALID_INPUT;
  delete ctx->open_batch;
  for (slm_batch* b : ctx->submitted) delete b;
  destroy_device(ctx);
  delete ctx;
  return SLM_OK;
}

const char* slm_last_error(const slm_ctx* ctx) {
  return ctx ? ctx->err.c_str() : g_create_error.c_str();
}

slm_status slm_device_bytes(const slm_ctx* ctx, int64_t* bytes) {
  if (!ctx || !bytes) return SLM_ERR_INVALID_INPUT;
  *bytes = ctx->device_bytes;
  return SLM_OK;
}

slm_status slm_launch_count(const slm_ctx* ctx, int64_t* launches) {
  if (!ctx || !launches) return SLM_ERR_INVALID_INPUT;
  *launches = ctx->launches;
  return SLM_OK;
}

// ---- sequences -------------------------------------------------------------

slm_status slm_seq_create(slm_ctx* ctx, int32_t max_sequence_length, int32_t* seq_id) {
  if (!ctx || !seq_id) return SLM_ERR_INVALID_INPUT;
  if (max_sequence_length <= 0 || max_sequence_length > ctx->cfg.context_length)
    return fail(ctx, SLM_ERR_INVALID_CONFIGURATION,
                "invalid model configuration: KV-cache max_sequence_length must be in 1..=%d",
                ctx->cfg.context_length);
  if (ctx->free_slots.empty())
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache",
                       "all %d sequence slots are in use", ctx->cfg.max_sequences);
  const int32_t id = ctx->free_slots.back();
  ctx->free_slots.pop_back();
  Seq& s = ctx->seqs[id];
  s.live = true;
  s.max_len = max_sequence_length;
  s.layer_len.assign(ctx->cfg.num_layers, 0);
  s.blocks.clear();
  s.in_batch = false;
  *seq_id = id;
  return SLM_OK;
}

slm_status slm_seq_free(slm_ctx* ctx, int32_t seq_id) {
  if (!ctx) return SLM_ERR_INVALID_INPUT;
  Seq* s = get_seq(ctx, seq_id);
  if (!s) return unknown_seq(ctx, seq_id);
  if (s->in_batch)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache",
                       "sequence %d belongs to an open batch", seq_id);
  if (s->in_flight)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache",
                       "sequence %d has a submitted step; wait for it first", seq_id);
  release_tail(ctx, seq_id, 0);
  s->live = false;
  s->layer_len.clear();
  ctx->free_slots.push_back(seq_id);
  return SLM_OK;
}

slm_status slm_seq_layer_length(const slm_ctx* ctx, int32_t seq_id, int32_t layer, int32_t* length) {
  if (!ctx || !length) return SLM_ERR_INVALID_INPUT;
  slm_ctx* mc = const_cast<slm_ctx*>(ctx);
  const Seq* s = get_seq(ctx, seq_id);
  if (!s) return unknown_seq(mc, seq_id);
  if (layer < 0 || layer >= ctx->cfg.num_layers)
    return input_error(mc, SLM_ERR_INVALID_INPUT, "KV cache", "layer index %d is outside 0..%d",
                       layer, ctx->cfg.num_layers);
  *length = s->layer_len[layer];
  return SLM_OK;
}

slm_status slm_seq_length(const slm_ctx* ctx, int32_t seq_id, int32_t* length) {
  if (!ctx || !length) return SLM_ERR_INVALID_INPUT;
  const Seq* s = get_seq(ctx, seq_id);
  if (!s) return unknown_seq(const_cast<slm_ctx*>(ctx), seq_id);
  *length = seq_min_len(*s);
  return SLM_OK;
}

slm_status slm_seq_is_empty(const slm_ctx* ctx, int32_t seq_id, int32_t* is_empty) {
  if (!ctx || !is_empty) return SLM_ERR_INVALID_INPUT;
  const Seq* s = get_seq(ctx, seq_id);
  if (!s) return unknown_seq(const_cast<slm_ctx*>(ctx), seq_id);
  *is_empty = seq_max_len(*s) == 0;
  return SLM_OK;
}

slm_status slm_seq_is_synchronized(const slm_ctx* ctx, int32_t seq_id, int32_t* is_sync) {
  if (!ctx || !is_sync) return SLM_ERR_INVALID_INPUT;
  const Seq* s = get_seq(ctx, seq_id);
  if (!s) return unknown_seq(const_cast<slm_ctx*>(ctx), seq_id);
  *is_sync = seq_synchronized(*s);
  return SLM_OK;
}

slm_status slm_seq_remaining_capacity(const slm_ctx* ctx, int32_t seq_id, int32_t* remaining) {
  if (!ctx || !remaining) return SLM_ERR_INVALID_INPUT;
  const Seq* s = get_seq(ctx, seq_id);
  if (!s) return unknown_seq(const_cast<slm_ctx*>(ctx), seq_id);
  *remaining = std::max(0, s->max_len - seq_max_len(*s));
  return SLM_OK;
}

slm_status slm_seq_truncate_all(slm_ctx* ctx, int32_t seq_id, int32_t length) {
  if (!ctx) return SLM_ERR_INVALID_INPUT;
  Seq* s = get_seq(ctx, seq_id);
  if (!s) return unknown_seq(ctx, seq_id);
  if (s->in_batch)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache",
                       "sequence %d belongs to an open batch", seq_id);
  for (int32_t l = 0; l < ctx->cfg.num_layers; ++l)
    if (s->layer_len[l] < length || length < 0)
      return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache",
                         "cannot restore all layers to %d: layer %d has length %d", length, l,
                         s->layer_len[l]);
  for (auto& v : s->layer_len) v = length;
  release_tail(ctx, seq_id, blocks_for(length));
  return SLM_OK;
}

slm_status slm_seqs_truncate_all(slm_ctx* ctx, int32_t n, const int32_t* h_seq_ids,
                                 const int32_t* h_lengths) {
  if (!ctx || n < 0 || (n > 0 && (!h_seq_ids || !h_lengths))) return SLM_ERR_INVALID_INPUT;
  for (int32_t i = 0; i < n; ++i) {
    slm_status rc = slm_seq_truncate_all(ctx, h_seq_ids[i], h_lengths[i]);
    if (rc) return rc;
  }
  return SLM_OK;
}

slm_status slm_seq_truncate_layer(slm_ctx* ctx, int32_t seq_id, int32_t layer, int32_t length) {
  if (!ctx) return SLM_ERR_INVALID_INPUT;
  Seq* s = get_seq(ctx, seq_id);
  if (!s) return unknown_seq(ctx, seq_id);
  if (s->in_batch)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache",
                       "sequence %d belongs to an open batch", seq_id);
  if (layer < 0 || layer >= ctx->cfg.num_layers)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache", "layer index %d is outside 0..%d",
                       layer, ctx->cfg.num_layers);
  if (length > s->layer_len[layer] || length < 0)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache",
                       "cannot extend layer %d from %d to %d while truncating", layer,
                       s->layer_len[layer], length);
  s->layer_len[layer] = length;
  release_tail(ctx, seq_id, blocks_for(seq_max_len(*s)));
  return SLM_OK;
}

slm_status slm_seq_clear(slm_ctx* ctx, int32_t seq_id) {
  if (!ctx) return SLM_ERR_INVALID_INPUT;
  Seq* s = get_seq(ctx, seq_id);
  if (!s) return unknown_seq(ctx, seq_id);
  if (s->in_batch)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache",
                       "sequence %d belongs to an open batch", seq_id);
  for (auto& v : s->layer_len) v = 0;
  release_tail(ctx, seq_id, 0);
  return SLM_OK;
}

slm_status slm_seq_blocks(const slm_ctx* ctx, int32_t seq_id, int32_t* h_ids, int32_t capacity,
                          int32_t* n_blocks) {
  if (!ctx || !n_blocks) return SLM_ERR_INVALID_INPUT;
  const Seq* s = get_seq(ctx, seq_id);
  if (!s) return unknown_seq(const_cast<slm_ctx*>(ctx), seq_id);
  *n_blocks = static_cast<int32_t>(s->blocks.size());
  for (int32_t i = 0; i < std::min(*n_blocks, capacity); ++i) h_ids[i] = s->blocks[i];
  return SLM_OK;
}

// ---- single-sequence operations -----------------------------------------------

slm_status slm_append_layer(slm_ctx* ctx, int32_t seq_id, int32_t layer, const float* d_keys,
                            const float* d_values, int32_t token_count, int32_t rotate_keys,
                            slm_stream stream) {
  if (!ctx) return SLM_ERR_INVALID_INPUT;
  slm_status rc = need_device(ctx);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Seq* q = get_seq(ctx, seq_id);
  if (!q) return unknown_seq(ctx, seq_id);
  if (q->in_batch)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache",
                       "sequence %d belongs to an open batch", seq_id);
  if (token_count <= 0 || !d_keys || !d_values)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV-cache keys",
                       "matrix dimensions must be greater than zero");
  if (layer < 0 || layer >= ctx->cfg.num_layers)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache", "layer index %d is outside 0..%d",
                       layer, ctx->cfg.num_layers);
  const int32_t cur = q->layer_len[layer];
  const int64_t new_len = static_cast<int64_t>(cur) + token_count;
  if (new_len > q->max_len)
    return input_error(ctx, SLM_ERR_CAPACITY, "KV cache",
                       "layer %d would grow to %lld tokens, exceeding capacity %d", layer,
                       static_cast<long long>(new_len), q->max_len);
  Undo undo;
  undo.updates_mark = ctx->pending_updates.size();
  undo.copies_mark = ctx->pending_copies.size();
  if (!reserve_positions(ctx, seq_id, cur, static_cast<int32_t>(new_len), undo)) {
    rollback_reserve(ctx, undo);
    return input_error(ctx, SLM_ERR_POOL_EXHAUSTED, "KV cache", "no free block in the pool");
  }
  std::vector<SeqEntry> e(1);
  e[0] = SeqEntry{seq_id, cur, token_count, 0, static_cast<int32_t>(new_len), {0, 0, 0}};
  StepDev dev;
  rc = upload_step(ctx, ctx->up_aux, s, e, nullptr, &dev);
  if (rc) {
    rollback_reserve(ctx, undo);
    return rc;
  }
  SeqEntry* d_seqs = dev.seqs;
  int32_t* d_status = dev.status;
  AppendLaunch a{};
  a.g = ctx->geom();
  a.layer = layer;
  a.seqs = d_seqs;
  a.n_seq = 1;
  a.total_tokens = token_count;
  a.k_in = d_keys;
  a.v_in = d_values;
  a.rotate = rotate_keys != 0;
  a.status = d_status;
  ctx->prev_decode_layer = -1;
  CU(ctx, launch_append(a, s));
  ++ctx->launches;
  int32_t status = 0;
  rc = finish_single(ctx, s, d_status, &status);
  if (rc) return rc;
  if (status & kStatusNonFinite) {
    // Nothing became visible: the length was never advanced. Blocks taken for
    // the new positions go back to the pool.
    release_tail(ctx, seq_id, blocks_for(seq_max_len(*q)));
    return input_error(ctx, SLM_ERR_NON_FINITE, "KV cache",
                       "all appended key/value values must be finite");
  }
  q->layer_len[layer] = static_cast<int32_t>(new_len);
  return SLM_OK;
}

slm_status slm_gather_layer(slm_ctx* ctx, int32_t seq_id, int32_t layer, float* d_keys,
                            float* d_values, slm_stream stream) {
  if (!ctx) return SLM_ERR_INVALID_INPUT;
  slm_status rc = need_device(ctx);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Seq* q = get_seq(ctx, seq_id);
  if (!q) return unknown_seq(ctx, seq_id);
  if (layer < 0 || layer >= ctx->cfg.num_layers)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache", "layer index %d is outside 0..%d",
                       layer, ctx->cfg.num_layers);
  rc = flush_excess(ctx, s, 0, 0);
  if (rc) return rc;
  GatherLaunch gl{};
  gl.g = ctx->geom();
  gl.layer = layer;
  gl.slot = seq_id;
  gl.length = q->layer_len[layer];
  gl.k_out = d_keys;
  gl.v_out = d_values;
  ctx->prev_decode_layer = -1;
  CU(ctx, launch_gather(gl, s));
  ++ctx->launches;
  return SLM_OK;
}

slm_status slm_attend_cached_query(slm_ctx* ctx, int32_t seq_id, int32_t layer,
                                   const float* d_query, float* d_out, slm_stream stream) {
  if (!ctx) return SLM_ERR_INVALID_INPUT;
  slm_status rc = need_device(ctx);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Seq* q = get_seq(ctx, seq_id);
  if (!q) return unknown_seq(ctx, seq_id);
  if (layer < 0 || layer >= ctx->cfg.num_layers)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache", "layer index %d is outside 0..%d",
                       layer, ctx->cfg.num_layers);
  if (!d_query || !d_out || !aligned16(d_query) || !aligned16(d_out))
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "cached attention",
                       "query and output buffers must be non-null and 16-byte aligned");
  const int32_t L = q->layer_len[layer];
  if (L == 0)  // attention.rs:690-695
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "cached attention",
                       "at least one cached key/value position is required");
  std::vector<SeqEntry> e(1);
  e[0] = SeqEntry{seq_id, L, 0, 0, L, {0, 0, 0}};
  StreamPlan plan;
  build_stream_plan(ctx, e, ctx->n_warps, plan);
  StepDev dev;
  rc = upload_step(ctx, ctx->up_aux, s, e, &plan, &dev);
  if (rc) return rc;
  StreamDecodeLaunch p = decode_launch(ctx, layer, dev, plan);
  p.q[0] = d_query;
  p.out[0] = d_out;
  p.fused = 0;
  ctx->prev_decode_layer = -1;
  CU(ctx, launch_decode(p, s));
  ++ctx->launches;
  // softmax_rows (attention.rs:731) fails on a non-finite score: the call
  // waits for the kernel and reports it as the reference's InvalidInput.
  int32_t status = 0;
  rc = finish_single(ctx, s, dev.status, &status);
  if (rc) return rc;
  if (status & kStatusNonFiniteScore)
    return input_error(ctx, SLM_ERR_NON_FINITE, "softmax", "all input values must be finite");
  return SLM_OK;
}

// ---- batches ------------------------------------------------------------------

slm_status slm_batch_begin(slm_ctx* ctx, int32_t n, const int32_t* h_seq_ids,
                           const int32_t* h_token_counts, slm_stream stream, slm_batch** out) {
  if (!ctx || !out) return SLM_ERR_INVALID_INPUT;
  *out = nullptr;
  slm_status rc = need_device(ctx);
  if (rc) return rc;
  if (ctx->open_batch)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "a batch is already open");
  if (n <= 0 || n > ctx->cfg.max_sequences || !h_seq_ids || !h_token_counts)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "batch size %d is outside 1..=%d", n,
                       ctx->cfg.max_sequences);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The step descriptor region is reused: a step on another stream than the
  // last submitted one starts after that one's kernels.
  if (!ctx->submitted.empty() && ctx->submitted.back()->stream != s) {
    const cudaError_t e = cudaStreamWaitEvent(s, ctx->rb_ev[ctx->submitted.back()->rb_slot], 0);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "slm_batch_begin");
  }
  // Validate everything before mutating anything.
  auto unmark = [&](int32_t upto) {
    for (int32_t i = 0; i < upto; ++i) ctx->seqs[h_seq_ids[i]].in_batch = false;
  };
  for (int32_t i = 0; i < n; ++i) {
    const int32_t id = h_seq_ids[i];
    Seq* q = get_seq(ctx, id);
    if (!q) {
      unmark(i);
      return unknown_seq(ctx, id);
    }
    if (q->in_batch) {
      unmark(i);
      return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch",
                         "sequence %d is already in a batch or appears twice", id);
    }
    q->in_batch = true;  // duplicate detection; undone below on every failure
  }
  auto clear_marks = [&] { unmark(n); };
  for (int32_t i = 0; i < n; ++i) {
    const Seq& q = ctx->seqs[h_seq_ids[i]];
    if (h_token_counts[i] <= 0) {
      clear_marks();
      return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch",
                         "sequence %d: token count must be greater than zero", h_seq_ids[i]);
    }
    if (!seq_synchronized(q)) {  // model.rs:345-350
      clear_marks();
      return input_error(ctx, SLM_ERR_INVALID_INPUT, "model cached decode",
                         "all cache layers must have the same length before decoding");
    }
    const int64_t nl = static_cast<int64_t>(q.layer_len[0]) + h_token_counts[i];
    if (nl > q.max_len) {  // kv_cache.rs:203-211
      clear_marks();
      return input_error(ctx, SLM_ERR_CAPACITY, "KV cache",
                         "sequence %d would grow to %lld tokens, exceeding capacity %d",
                         h_seq_ids[i], static_cast<long long>(nl), q.max_len);
    }
  }
  Undo undo;
  undo.updates_mark = ctx->pending_updates.size();
  undo.copies_mark = ctx->pending_copies.size();
  std::unique_ptr<slm_batch> b(new slm_batch());
  b->ctx = ctx;
  b->stream = s;
  b->seq_ids.assign(h_seq_ids, h_seq_ids + n);
  b->counts.assign(h_token_counts, h_token_counts + n);
  b->base.resize(n);
  std::vector<SeqEntry> entries(n);
  int32_t row = 0;
  for (int32_t i = 0; i < n; ++i) {
    const int32_t id = h_seq_ids[i];
    const int32_t base = ctx->seqs[id].layer_len[0];
    if (!reserve_positions(ctx, id, base, base + h_token_counts[i], undo)) {
      rollback_reserve(ctx, undo);
      clear_marks();
      return input_error(ctx, SLM_ERR_POOL_EXHAUSTED, "KV cache", "no free block in the pool");
    }
    b->base[i] = base;
    entries[i] = SeqEntry{id, base, h_token_counts[i], row, base + h_token_counts[i], {0, 0, 0}};
    row += h_token_counts[i];
    b->max_count = std::max(b->max_count, h_token_counts[i]);
  }
  b->total_tokens = row;
  // A decode step (one token each) carries its decode plan in the same upload.
  StreamPlan& plan = ctx->plan;
  const bool decode = (b->max_count == 1);
  if (decode) {
    build_stream_plan(ctx, entries, ctx->n_warps, plan);
    b->n_pairs = static_cast<int32_t>(plan.pairs.size());
    b->total_blocks = static_cast<int32_t>(plan.chunks.size());
  }
  // The decode kernel reads the chunk stream, not the device block table, so
  // a decode step leaves pure table writes pending (copies are applied now);
  // every kernel that reads the table flushes them first.
  b->up_slot = ctx->up_batch.next;
  rc = upload_step(ctx, ctx->up_batch, s, entries, decode ? &plan : nullptr, &b->dev,
                   /*with_table_updates=*/!decode);
  if (rc) {
    rollback_reserve(ctx, undo);
    clear_marks();
    return rc;
  }
  b->layer_done.assign(ctx->cfg.num_layers, 0);
  ctx->open_batch = b.get();
  *out = b.release();
  return SLM_OK;
}

namespace {
slm_status batch_layer_check(slm_batch* b, int32_t layer) {
  slm_ctx* ctx = b->ctx;
  if (ctx->open_batch != b)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "the batch is not open");
  if (layer < 0 || layer >= ctx->cfg.num_layers)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache", "layer index %d is outside 0..%d",
                       layer, ctx->cfg.num_layers);
  return need_device(ctx);
}
}  // namespace

namespace {
// Checks one decode layer's arguments (the batch open, every count 1, the
// layer not yet appended, the buffers non-null and 16-byte aligned).
slm_status decode_layer_check(slm_batch* b, int32_t layer, const float* d_query,
                              const float* d_keys, const float* d_values, const float* d_out) {
  slm_ctx* ctx = b->ctx;
  slm_status rc = batch_layer_check(b, layer);
  if (rc) return rc;
  if (b->max_count != 1)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch",
                       "decode layers need exactly one new token per sequence");
  if (b->layer_done[layer])
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "layer %d was already appended", layer);
  if (!d_query || !d_keys || !d_values || !d_out)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "null tensor");
  if (!aligned16(d_query) || !aligned16(d_keys) || !aligned16(d_values) || !aligned16(d_out))
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch",
                       "query, key, value and output buffers must be 16-byte aligned");
  return SLM_OK;
}

// Launches the decode of layers first .. first + nl - 1 (io[i] for layer
// first + i) as one kernel, then advances those layers' lengths.
slm_status decode_launch_layers(slm_batch* b, int32_t first, int32_t nl, const slm_layer_io* io,
                                uint32_t* out_bf16 = nullptr) {
  slm_ctx* ctx = b->ctx;
  StreamDecodeLaunch p = decode_launch(ctx, first, b->dev, ctx->plan);
  p.n_layers = nl;
  p.out_bf16 = nl == 1 ? out_bf16 : nullptr;
  for (int32_t i = 0; i < nl; ++i) {
    p.q[i] = io[i].query;
    p.k_new[i] = io[i].keys;
    p.v_new[i] = io[i].values;
    p.out[i] = io[i].out;
  }
  p.fused = 1;
  // The first stages may be fetched early when the previous launch was a
  // decode of other layers only.
  const int32_t last = first + nl - 1;
  p.early_kv = (ctx->prev_decode_layer >= 0 &&
                (last < ctx->prev_decode_layer || first > ctx->prev_decode_last)) ? 1 : 0;
  ctx->prev_decode_layer = first;
  ctx->prev_decode_last = last;
  CU(ctx, launch_decode(p, b->stream));
  ++ctx->launches;
  for (int32_t layer = first; layer <= last; ++layer) {
    b->layer_done[layer] = 1;
    for (size_t i = 0; i < b->seq_ids.size(); ++i)
      ctx->seqs[b->seq_ids[i]].layer_len[layer] = b->base[i] + b->counts[i];
  }
  return SLM_OK;
}

bool ranges_overlap(const void* a, size_t na, const void* b, size_t nb) {
  const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return x < y + nb && y < x + na;
}
}  // namespace

slm_status slm_batch_decode_layer(slm_batch* b, int32_t layer, const float* d_query,
                                  const float* d_keys, const float* d_values, float* d_out) {
  if (!b) return SLM_ERR_INVALID_INPUT;
  slm_status rc = decode_layer_check(b, layer, d_query, d_keys, d_values, d_out);
  if (rc) return rc;
  const slm_layer_io io{d_query, d_keys, d_values, d_out};
  return decode_launch_layers(b, layer, 1, &io);
}

extern "C++" {
namespace slmkv {
slm_status batch_decode_layer_bf16(slm_batch* b, int32_t layer, const float* d_query,
                                   const float* d_keys, const float* d_values, float* d_out,
                                   uint32_t* d_out_bf16) {
  if (!b) return SLM_ERR_INVALID_INPUT;
  slm_status rc = decode_layer_check(b, layer, d_query, d_keys, d_values, d_out);
  if (rc) return rc;
  const slm_layer_io io{d_query, d_keys, d_values, d_out};
  return decode_launch_layers(b, layer, 1, &io, d_out_bf16);
}
}  // namespace slmkv
}

slm_status slm_batch_decode_layers(slm_batch* b, int32_t first_layer, int32_t n_layers,
                                   const slm_layer_io* io) {
  if (!b) return SLM_ERR_INVALID_INPUT;
  slm_ctx* ctx = b->ctx;
  if (n_layers <= 0 || !io)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch",
                       "a layer count of at least 1 and its buffers are required");
  if (first_layer < 0 || n_layers > ctx->cfg.num_layers - first_layer)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache",
                       "layers %d..%d are outside 0..%d", first_layer,
                       first_layer + n_layers - 1, ctx->cfg.num_layers);
  // Everything is checked before the first launch.
  for (int32_t i = 0; i < n_layers; ++i) {
    const slm_status rc = decode_layer_check(b, first_layer + i, io[i].query, io[i].keys,
                                             io[i].values, io[i].out);
    if (rc) return rc;
  }
  // The layers of one launch run at the same time: a layer's output may not
  // overlap another layer's inputs or output.
  const size_t n = b->seq_ids.size();
  const size_t qb = n * ctx->cfg.num_query_heads * kHeadDim * sizeof(float);
  const size_t kvb = n * ctx->cfg.num_key_value_heads * kHeadDim * sizeof(float);
  for (int32_t i = 0; i < n_layers; ++i)
    for (int32_t j = 0; j < n_layers; ++j) {
      if (i == j) continue;
      const void* o = io[i].out;
      if (ranges_overlap(o, qb, io[j].query, qb) || ranges_overlap(o, qb, io[j].keys, kvb) ||
          ranges_overlap(o, qb, io[j].values, kvb) || ranges_overlap(o, qb, io[j].out, qb))
        return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch",
                           "layer %d's output overlaps layer %d's buffers", first_layer + i,
                           first_layer + j);
    }
  // One launch runs up to kMaxLaunchLayers layers of an f32 pool when every
  // warp's slice fits its 32-entry windows; otherwise one launch per layer.
  const int32_t per =
      (ctx->plan.fits_window && ctx->cfg.kv_dtype == SLM_KV_F32) ? ctx->launch_layers : 1;
  for (int32_t i = 0; i < n_layers; i += per) {
    const slm_status rc = decode_launch_layers(b, first_layer + i, std::min(per, n_layers - i), io + i);
    if (rc) return rc;
  }
  return SLM_OK;
}

namespace {
// Grows the host-IO staging to `in` / `out` floats a slot (waits for the
// device first: a slot may be in use).
slm_status host_io_reserve(slm_ctx* c, size_t in, size_t out) {
  slm_ctx::HostIo& io = c->io;
  if (!io.h2d) {
    CU(c, cudaStreamCreateWithFlags(&io.h2d, cudaStreamNonBlocking));
    for (int k = 0; k < kUploadSlots; ++k)
      for (cudaEvent_t* ev : {&io.in_done[k], &io.used[k], &io.read[k]})
        CU(c, cudaEventCreateWithFlags(ev, cudaEventDisableTiming));
  }
  if (in <= io.in_cap && out <= io.out_cap) return SLM_OK;
  CU(c, cudaDeviceSynchronize());
  for (int k = 0; k < kUploadSlots; ++k) {
    if (io.d_in[k]) cudaFree(io.d_in[k]);
    if (io.d_out[k]) cudaFree(io.d_out[k]);
    io.d_in[k] = io.d_out[k] = nullptr;
  }
  c->device_bytes -= static_cast<int64_t>((io.in_cap + io.out_cap) * sizeof(float)) * kUploadSlots;
  io.in_cap = io.out_cap = 0;
  for (int k = 0; k < kUploadSlots; ++k) {
    CU(c, cudaMalloc(reinterpret_cast<void**>(&io.d_in[k]), in * sizeof(float)));
    CU(c, cudaMalloc(reinterpret_cast<void**>(&io.d_out[k]), out * sizeof(float)));
  }
  io.in_cap = in;
  io.out_cap = out;
  c->device_bytes += static_cast<int64_t>((in + out) * sizeof(float)) * kUploadSlots;
  return SLM_OK;
}
}  // namespace

slm_status slm_batch_decode_layers_host(slm_batch* b, int32_t first_layer, int32_t n_layers,
                                        const float* h_query, const float* h_keys,
                                        const float* h_values, float* h_out) {
  if (!b) return SLM_ERR_INVALID_INPUT;
  slm_ctx* ctx = b->ctx;
  if (n_layers <= 0 || n_layers > ctx->cfg.num_layers || !h_query || !h_keys || !h_values || !h_out)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch",
                       "a layer count of at least 1 and host buffers are required");
  slm_status rc = batch_layer_check(b, first_layer);
  if (rc) return rc;
  if (first_layer + n_layers > ctx->cfg.num_layers)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache", "layers %d..%d are outside 0..%d",
                       first_layer, first_layer + n_layers - 1, ctx->cfg.num_layers);
  const size_t n = b->seq_ids.size();
  const size_t qn = n * ctx->cfg.num_query_heads * kHeadDim;
  const size_t kvn = n * ctx->cfg.num_key_value_heads * kHeadDim;
  const size_t L = static_cast<size_t>(n_layers);
  if ((rc = host_io_reserve(ctx, L * (qn + 2 * kvn), L * qn))) return rc;
  slm_ctx::HostIo& io = ctx->io;
  const int k = b->up_slot;
  float* dq = io.d_in[k];
  float* dk = dq + L * qn;
  float* dv = dk + L * kvn;
  float* dout = io.d_out[k];
  std::vector<slm_layer_io> lio(L);
  for (size_t i = 0; i < L; ++i) lio[i] = slm_layer_io{dq + i * qn, dk + i * kvn, dv + i * kvn, dout + i * qn};
  // every layer's arguments checked before anything is queued
  for (int32_t i = 0; i < n_layers; ++i)
    if ((rc = decode_layer_check(b, first_layer + i, lio[i].query, lio[i].keys, lio[i].values,
                                 lio[i].out)))
      return rc;
  // inputs in, after the kernels that last read this slot
  CU(ctx, cudaStreamWaitEvent(io.h2d, io.used[k], 0));
  if (h_keys == h_query + L * qn && h_values == h_keys + L * kvn) {  // one host block: one copy
    CU(ctx, cudaMemcpyAsync(dq, h_query, L * (qn + 2 * kvn) * sizeof(float), cudaMemcpyHostToDevice,
                            io.h2d));
  } else {
    CU(ctx, cudaMemcpyAsync(dq, h_query, L * qn * sizeof(float), cudaMemcpyHostToDevice, io.h2d));
    CU(ctx, cudaMemcpyAsync(dk, h_keys, L * kvn * sizeof(float), cudaMemcpyHostToDevice, io.h2d));
    CU(ctx, cudaMemcpyAsync(dv, h_values, L * kvn * sizeof(float), cudaMemcpyHostToDevice, io.h2d));
  }
  CU(ctx, cudaEventRecord(io.in_done[k], io.h2d));
  // the step's kernels, after its inputs and after this slot's last outputs left
  CU(ctx, cudaStreamWaitEvent(b->stream, io.in_done[k], 0));
  CU(ctx, cudaStreamWaitEvent(b->stream, io.read[k], 0));
  if ((rc = slm_batch_decode_layers(b, first_layer, n_layers, lio.data()))) return rc;
  CU(ctx, cudaEventRecord(io.used[k], b->stream));
  // outputs out on the readback stream, ahead of the step's statuses, so the
  // batch's end / wait returns after they are on the host
  CU(ctx, cudaStreamWaitEvent(ctx->readback_stream, io.used[k], 0));
  CU(ctx, cudaMemcpyAsync(h_out, dout, L * qn * sizeof(float), cudaMemcpyDeviceToHost,
                          ctx->readback_stream));
  CU(ctx, cudaEventRecord(io.read[k], ctx->readback_stream));
  return SLM_OK;
}

slm_status slm_batch_append_layer(slm_batch* b, int32_t layer, const float* d_keys,
                                  const float* d_values, int32_t rotate_keys) {
  if (!b) return SLM_ERR_INVALID_INPUT;
  slm_ctx* ctx = b->ctx;
  slm_status rc = batch_layer_check(b, layer);
  if (rc) return rc;
  if (b->layer_done[layer])
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "layer %d was already appended", layer);
  if (!d_keys || !d_values) return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "null tensor");
  rc = flush_excess(ctx, b->stream, 0, 0);  // the append reads the device block table
  if (rc) return rc;
  AppendLaunch a{};
  a.g = ctx->geom();
  a.layer = layer;
  a.seqs = b->dev.seqs;
  a.n_seq = static_cast<int32_t>(b->seq_ids.size());
  a.total_tokens = b->total_tokens;
  a.k_in = d_keys;
  a.v_in = d_values;
  a.rotate = rotate_keys != 0;
  a.status = b->dev.status;
  ctx->prev_decode_layer = -1;
  CU(ctx, launch_append(a, b->stream));
  ++ctx->launches;
  b->layer_done[layer] = 1;
  for (size_t i = 0; i < b->seq_ids.size(); ++i)
    ctx->seqs[b->seq_ids[i]].layer_len[layer] = b->base[i] + b->counts[i];
  return SLM_OK;
}

slm_status slm_batch_prefill_attention(slm_batch* b, int32_t layer, const float* d_query,
                                       int32_t rotate_query, float* d_out) {
  if (!b) return SLM_ERR_INVALID_INPUT;
  slm_ctx* ctx = b->ctx;
  slm_status rc = batch_layer_check(b, layer);
  if (rc) return rc;
  if (!b->layer_done[layer])
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "cached attention prefill",
                       "layer %d must be appended before its attention", layer);
  // bf16 pools run on the tensor cores (any supported group); the f32 kernel
  // keeps up to 4 query heads per KV head in shared memory.
  if (ctx->cfg.kv_dtype != SLM_KV_BF16 && ctx->group > 4)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "cached attention prefill",
                       "more than 4 query heads per KV head are not supported in f32 prefill");
  if (!d_query || !d_out) return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "null tensor");
  rc = flush_excess(ctx, b->stream, 0, 0);  // the prefill reads the device block table
  if (rc) return rc;
  PrefillLaunch p{};
  p.g = ctx->geom();
  p.layer = layer;
  p.seqs = b->dev.seqs;
  p.n_seq = static_cast<int32_t>(b->seq_ids.size());
  p.total_tokens = b->total_tokens;
  p.q = d_query;
  p.rotate = rotate_query != 0;
  p.out = d_out;
  p.max_count = b->max_count;
  p.status = b->dev.status;
  p.tmap_k = ctx->tmap_k;
  p.tmap_v = ctx->tmap_v;
  ctx->prev_decode_layer = -1;
  CU(ctx, launch_prefill(p, b->stream));
  ++ctx->launches;
  return SLM_OK;
}

slm_status slm_batch_decode_layer_exact(slm_batch* b, int32_t layer, const float* d_query,
                                        const float* d_keys, const float* d_values, float* d_out) {
  if (!b) return SLM_ERR_INVALID_INPUT;
  slm_ctx* ctx = b->ctx;
  slm_status rc = batch_layer_check(b, layer);
  if (rc) return rc;
  if (b->max_count != 1)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch",
                       "decode layers need exactly one new token per sequence");
  if (b->layer_done[layer])
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "layer %d was already appended", layer);
  if (ctx->cfg.kv_dtype != SLM_KV_F32)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "cached attention",
                       "exact-order attention needs an f32 pool");
  if (!d_query || !d_keys || !d_values || !d_out)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "null tensor");
  if (!aligned16(d_query) || !aligned16(d_keys) || !aligned16(d_values) || !aligned16(d_out))
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch",
                       "query, key, value and output buffers must be 16-byte aligned");
  int32_t max_ctx = 0;
  for (size_t i = 0; i < b->seq_ids.size(); ++i)
    max_ctx = std::max(max_ctx, b->base[i] + b->counts[i]);
  if (max_ctx > kExactMaxCtx)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "cached attention",
                       "exact-order attention takes at most %d positions, the batch reaches %d",
                       kExactMaxCtx, max_ctx);
  rc = flush_excess(ctx, b->stream, 0, 0);  // the kernel reads the device block table
  if (rc) return rc;
  PrefillLaunch p{};
  p.g = ctx->geom();
  p.layer = layer;
  p.seqs = b->dev.seqs;
  p.n_seq = static_cast<int32_t>(b->seq_ids.size());
  p.total_tokens = b->total_tokens;
  p.q = d_query;
  p.rotate = 1;
  p.out = d_out;
  p.max_count = 1;
  p.status = b->dev.status;
  p.max_ctx = max_ctx;
  p.k_new = d_keys;
  p.v_new = d_values;
  p.fused = 1;
  ctx->prev_decode_layer = -1;
  CU(ctx, launch_exact_attention(p, b->stream));
  ++ctx->launches;
  b->layer_done[layer] = 1;
  for (size_t i = 0; i < b->seq_ids.size(); ++i)
    ctx->seqs[b->seq_ids[i]].layer_len[layer] = b->base[i] + b->counts[i];
  return SLM_OK;
}

slm_status slm_batch_attention_exact(slm_batch* b, int32_t layer, const float* d_query,
                                     int32_t rotate_query, float* d_out) {
  if (!b) return SLM_ERR_INVALID_INPUT;
  slm_ctx* ctx = b->ctx;
  slm_status rc = batch_layer_check(b, layer);
  if (rc) return rc;
  if (!b->layer_done[layer])
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "cached attention",
                       "layer %d must be appended before its attention", layer);
  if (ctx->cfg.kv_dtype != SLM_KV_F32)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "cached attention",
                       "exact-order attention needs an f32 pool");
  if (!d_query || !d_out) return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "null tensor");
  int32_t max_ctx = 0;
  for (size_t i = 0; i < b->seq_ids.size(); ++i)
    max_ctx = std::max(max_ctx, b->base[i] + b->counts[i]);
  if (max_ctx > kExactMaxCtx)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "cached attention",
                       "exact-order attention takes at most %d positions, the batch reaches %d",
                       kExactMaxCtx, max_ctx);
  rc = flush_excess(ctx, b->stream, 0, 0);  // the kernel reads the device block table
  if (rc) return rc;
  PrefillLaunch p{};
  p.g = ctx->geom();
  p.layer = layer;
  p.seqs = b->dev.seqs;
  p.n_seq = static_cast<int32_t>(b->seq_ids.size());
  p.total_tokens = b->total_tokens;
  p.q = d_query;
  p.rotate = rotate_query != 0;
  p.out = d_out;
  p.max_count = b->max_count;
  p.status = b->dev.status;
  p.max_ctx = max_ctx;
  ctx->prev_decode_layer = -1;
  CU(ctx, launch_exact_attention(p, b->stream));
  ++ctx->launches;
  return SLM_OK;
}

namespace {
// Rolls sequence `id` back to at most `target` tokens in every layer and
// forces the same rollback on every later batch (submitted or open) that
// holds it: those were planned on the lengths this rollback undoes.
void roll_back_seq(slm_ctx* ctx, const slm_batch* from, int32_t id, int32_t target, int32_t code) {
  Seq& q = ctx->seqs[id];
  for (auto& v : q.layer_len) v = std::min(v, target);
  release_tail(ctx, id, blocks_for(seq_max_len(q)));
  bool later = false;
  auto poison = [&](slm_batch* m) {
    for (size_t j = 0; j < m->seq_ids.size(); ++j)
      if (m->seq_ids[j] == id) {
        if (m->poison_base[j] < 0 || target < m->poison_base[j]) m->poison_base[j] = target;
        if (!m->poison_code[j]) m->poison_code[j] = code;
      }
  };
  for (slm_batch* m : ctx->submitted) {
    if (m == from) {
      later = true;
      continue;
    }
    if (later && !m->resolved) poison(m);
  }
  if (ctx->open_batch && ctx->open_batch != from) poison(ctx->open_batch);
}

// Drops an open batch (slm_batch_rollback, or a failed submit): every
// sequence back to its begin length.
void batch_discard(slm_batch* b) {
  slm_ctx* ctx = b->ctx;
  if (has_device(ctx)) cudaEventRecord(ctx->up_batch.consumed[b->up_slot], b->stream);
  for (size_t i = 0; i < b->seq_ids.size(); ++i) {
    ctx->seqs[b->seq_ids[i]].in_batch = false;
    roll_back_seq(ctx, b, b->seq_ids[i], b->base[i], SLM_ERR_INVALID_INPUT);
  }
  ctx->open_batch = nullptr;
  delete b;
}

// Resolves the oldest submitted batch: waits for its status readback, sets
// each sequence's status and rolls failed sequences back
// (model.rs:390-396), in submission order.
void resolve_oldest(slm_ctx* ctx) {
  slm_batch* b = ctx->submitted.front();
  const size_t n = b->seq_ids.size();
  const int32_t* rb = ctx->h_rb + static_cast<size_t>(b->rb_slot) * (ctx->cfg.max_sequences + 2);
  const cudaError_t e = cudaEventSynchronize(ctx->rb_ev[b->rb_slot]);
  slm_status dev = SLM_OK;
  std::string dev_msg;
  if (e != cudaSuccess) {
    dev = SLM_ERR_CUDA;
    dev_msg = std::string("CUDA error in slm_batch_wait: ") + cudaGetErrorString(e);
  } else if (rb[0]) {
    const int32_t w = rb[0];
    cudaMemsetAsync(ctx->d_error, 0, sizeof(int32_t), b->stream);
    cudaMemsetAsync(ctx->d_counters, 0, ctx->counter_bytes(), b->stream);
    char buf[160];
    if (w & kErrTimeout) {
      dev = SLM_ERR_DEVICE_TIMEOUT;
      snprintf(buf, sizeof buf, "device wait timed out (error word 0x%x)", w);
    } else if (w & kErrLayout) {
      dev = SLM_ERR_CUDA;
      snprintf(buf, sizeof buf, "CUDA error: a kernel found its shared memory misaligned (0x%x)", w);
    } else if (w & kErrBadToken) {
      dev = SLM_ERR_INVALID_INPUT;  // embedding.rs:36-43
      snprintf(buf, sizeof buf, "invalid input for embedding lookup: token id outside the vocabulary (0x%x)", w);
    } else if (w & kErrLogits) {
      dev = SLM_ERR_INVALID_INPUT;  // greedy.rs argmax_finite
      snprintf(buf, sizeof buf, "invalid input for greedy decoding: final-position logits are not finite (0x%x)", w);
    } else {
      dev = SLM_ERR_INVALID_INPUT;
      snprintf(buf, sizeof buf,
               "invalid input for KV cache: block table held an out-of-pool id (0x%x)", w);
    }
    dev_msg = buf;
  }
  b->codes.assign(n, SLM_OK);
  int32_t first_bits = 0;  // status bits of the first sequence that failed
  for (size_t i = 0; i < n; ++i) {
    const int32_t st = (dev == SLM_OK) ? rb[2 + i] : 0;
    int32_t code = SLM_OK;
    if (dev != SLM_OK) code = dev;
    else if (b->poison_base[i] >= 0) code = b->poison_code[i];
    else if (st & (kStatusNonFinite | kStatusNonFiniteScore)) code = SLM_ERR_NON_FINITE;
    else if (!b->complete[i]) code = SLM_ERR_INVALID_INPUT;
    b->codes[i] = code;
    if (code != SLM_OK && b->first == SLM_OK) {
      b->first = code;
      first_bits = st;
    }
  }
  for (size_t i = 0; i < n; ++i) {
    const int32_t id = b->seq_ids[i];
    --ctx->seqs[id].in_flight;
    if (b->codes[i] != SLM_OK) {
      int32_t target = b->base[i];
      if (b->poison_base[i] >= 0) target = std::min(target, b->poison_base[i]);
      roll_back_seq(ctx, b, id, target, b->codes[i]);
    }
  }
  if (b->first == SLM_ERR_NON_FINITE && !(first_bits & kStatusNonFinite) &&
      (first_bits & kStatusNonFiniteScore))  // softmax.rs:17-22 through attention.rs:731
    b->msg = "invalid input for softmax: all input values must be finite";
  else if (b->first == SLM_ERR_NON_FINITE)
    b->msg = "invalid input for KV cache: all appended key/value values must be finite";
  else if (dev != SLM_OK)
    b->msg = dev_msg;
  else if (b->first == SLM_ERR_INVALID_INPUT)
    b->msg = "invalid input for model cached decode: all cache layers must advance by exactly "
             "one step";
  b->resolved = true;
  ctx->rb_busy[b->rb_slot] = false;
  ctx->submitted.pop_front();
}

slm_status submit(slm_batch* b, bool extra_slot) {
  slm_ctx* ctx = b->ctx;
  if (ctx->open_batch != b)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "the batch is not open");
  if (!extra_slot && ctx->submitted.size() >= static_cast<size_t>(kMaxInFlight))
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch",
                       "at most %d submitted batches may be pending; wait for one first",
                       kMaxInFlight);
  int slot = -1;
  for (int k = 0; k < kReadbackSlots && slot < 0; ++k)
    if (!ctx->rb_busy[k]) slot = k;
  const size_t n = b->seq_ids.size();
  cudaError_t e = cudaErrorNotReady;
  if (slot >= 0 && has_device(ctx)) {
    int32_t* rb = ctx->h_rb + static_cast<size_t>(slot) * (ctx->cfg.max_sequences + 2);
    // After the batch's kernels (which are then done with its descriptor)
    // the statuses come back on the readback stream.
    cudaStream_t cs = ctx->readback_stream;
    e = cudaEventRecord(ctx->up_batch.consumed[b->up_slot], b->stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, ctx->up_batch.consumed[b->up_slot], 0);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(rb + 2, b->dev.status, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(rb, ctx->d_error, sizeof(int32_t), cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess) e = cudaEventRecord(ctx->rb_ev[slot], cs);
  }
  if (e != cudaSuccess) {
    batch_discard(b);
    return slot < 0 ? input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "no readback slot free")
                    : cuda_fail(ctx, e, "slm_batch_submit");
  }
  b->complete.assign(n, 1);
  b->poison_base.assign(n, -1);
  b->poison_code.assign(n, 0);
  for (size_t i = 0; i < n; ++i) {
    Seq& q = ctx->seqs[b->seq_ids[i]];
    const int32_t want = b->base[i] + b->counts[i];
    for (int32_t v : q.layer_len) b->complete[i] = b->complete[i] && (v == want);
    q.in_batch = false;
    ++q.in_flight;
  }
  b->submitted = true;
  b->rb_slot = slot;
  ctx->rb_busy[slot] = true;
  ctx->open_batch = nullptr;
  ctx->submitted.push_back(b);
  return SLM_OK;
}
}  // namespace

slm_status slm_batch_submit(slm_batch* b) {
  if (!b) return SLM_ERR_INVALID_INPUT;
  return submit(b, false);
}

slm_status slm_batch_wait(slm_batch* b, int32_t* h_status) {
  if (!b) return SLM_ERR_INVALID_INPUT;
  slm_ctx* ctx = b->ctx;
  if (!b->submitted)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "batch", "the batch was not submitted");
  while (!b->resolved) resolve_oldest(ctx);
  if (h_status)
    for (size_t i = 0; i < b->codes.size(); ++i) h_status[i] = b->codes[i];
  const slm_status rc = b->first;
  if (rc != SLM_OK) ctx->err = b->msg;
  delete b;
  return rc;
}

slm_status slm_batch_end(slm_batch* b, int32_t* h_status) {
  if (!b) return SLM_ERR_INVALID_INPUT;
  const slm_status rc = submit(b, true);
  if (rc) return rc;
  return slm_batch_wait(b, h_status);
}

slm_status slm_batch_rollback(slm_batch* b) {
  if (!b) return SLM_ERR_INVALID_INPUT;
  if (b->ctx->open_batch != b)
    return input_error(b->ctx, SLM_ERR_INVALID_INPUT, "batch", "the batch is not open");
  batch_discard(b);
  return SLM_OK;
}

// ---- prefix cache -----------------------------------------------------------

namespace {
uint64_t chain_key(uint64_t parent_key, const uint32_t* toks) {
  uint64_t h = mix64(parent_key ^ 0x51ed27a3c6b9f1d5ull);
  for (int i = 0; i < kBlockTokens; ++i) h = mix64(h ^ toks[i]);
  return h;
}
int32_t find_indexed(const slm_ctx* c, uint64_t key, int32_t parent, const uint32_t* toks) {
  auto range = c->index.equal_range(key);
  for (auto it = range.first; it != range.second; ++it) {
    const BlockMeta& m = c->meta[it->second];
    if (m.parent == parent && std::equal(m.tokens.begin(), m.tokens.end(), toks))
      return it->second;
  }
  return -1;
}
}  // namespace

slm_status slm_prefix_attach(slm_ctx* ctx, int32_t seq_id, const uint32_t* h_tokens,
                             int32_t n_tokens, int32_t* reused_tokens) {
  if (!ctx || !reused_tokens) return SLM_ERR_INVALID_INPUT;
  *reused_tokens = 0;
  Seq* q = get_seq(ctx, seq_id);
  if (!q) return unknown_seq(ctx, seq_id);
  if (q->in_batch || seq_max_len(*q) != 0 || !q->blocks.empty())
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "prefix cache",
                       "a prefix can only be attached to an empty sequence");
  if (n_tokens < 0 || (n_tokens > 0 && !h_tokens))
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "prefix cache", "invalid token span");
  const int32_t limit = std::min(n_tokens, q->max_len) / kBlockTokens;
  uint64_t key = 0;
  int32_t parent = -1;
  std::vector<int32_t> chain;
  for (int32_t j = 0; j < limit; ++j) {
    const uint32_t* toks = h_tokens + static_cast<size_t>(j) * kBlockTokens;
    key = chain_key(key, toks);
    const int32_t b = find_indexed(ctx, key, parent, toks);
    if (b < 0) break;
    chain.push_back(b);
    parent = b;
  }
  ++ctx->clock;
  for (size_t j = 0; j < chain.size(); ++j) {
    const int32_t b = chain[j];
    ++ctx->refcount[b];
    ctx->meta[b].stamp = ctx->clock;
    q->blocks.push_back(b);
    ctx->pending_updates.push_back(TableUpdate{seq_id, static_cast<int32_t>(j), b, 0});
  }
  const int32_t reused = static_cast<int32_t>(chain.size()) * kBlockTokens;
  for (auto& v : q->layer_len) v = reused;
  *reused_tokens = reused;
  return SLM_OK;
}

slm_status slm_prefix_publish(slm_ctx* ctx, int32_t seq_id, const uint32_t* h_tokens,
                              int32_t n_tokens, int32_t* indexed_blocks) {
  if (!ctx) return SLM_ERR_INVALID_INPUT;
  Seq* q = get_seq(ctx, seq_id);
  if (!q) return unknown_seq(ctx, seq_id);
  if (!seq_synchronized(*q))
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "prefix cache",
                       "all cache layers must have the same length before publishing");
  if (n_tokens < 0 || n_tokens > seq_min_len(*q) || (n_tokens > 0 && !h_tokens))
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "prefix cache",
                       "%d tokens exceed the sequence length %d", n_tokens, seq_min_len(*q));
  const int32_t full = n_tokens / kBlockTokens;
  uint64_t key = 0;
  int32_t parent = -1;
  int32_t count = 0;
  ++ctx->clock;
  for (int32_t j = 0; j < full; ++j) {
    const uint32_t* toks = h_tokens + static_cast<size_t>(j) * kBlockTokens;
    key = chain_key(key, toks);
    int32_t b = find_indexed(ctx, key, parent, toks);
    if (b < 0) {
      b = q->blocks[j];
      BlockMeta& m = ctx->meta[b];
      if (m.indexed) break;  // this block already stands for another chain
      m.indexed = true;
      m.parent = parent;
      m.key = key;
      std::copy(toks, toks + kBlockTokens, m.tokens.begin());
      ctx->index.emplace(key, b);
      ++ctx->refcount[b];
      ++ctx->indexed_blocks;
    }
    ctx->meta[b].stamp = ctx->clock;
    parent = b;
    ++count;
  }
  if (indexed_blocks) *indexed_blocks = count;
  return SLM_OK;
}

slm_status slm_pool_stats(const slm_ctx* ctx, int32_t* free_blocks, int32_t* indexed_blocks) {
  if (!ctx) return SLM_ERR_INVALID_INPUT;
  if (free_blocks) *free_blocks = static_cast<int32_t>(ctx->free_list.size());
  if (indexed_blocks) *indexed_blocks = ctx->indexed_blocks;
  return SLM_OK;
}

slm_status slm_ctx_config(const slm_ctx* ctx, slm_config* out) {
  if (!ctx || !out) return SLM_ERR_INVALID_INPUT;
  *out = ctx->cfg;
  return SLM_OK;
}

slm_status slm_pool_shuffle(slm_ctx* ctx, uint64_t seed) {
  if (!ctx) return SLM_ERR_INVALID_INPUT;
  if (static_cast<int32_t>(ctx->free_list.size()) != ctx->cfg.num_blocks)
    return input_error(ctx, SLM_ERR_INVALID_INPUT, "KV cache",
                       "the pool can only be shuffled while no block is in use");
  std::mt19937_64 rng(seed);
  std::shuffle(ctx->free_list.begin(), ctx->free_list.end(), rng);
  return SLM_OK;
}

}  // extern "C"
