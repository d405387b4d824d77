// Allocation-free decode attention: slm_decode_attention_noalloc.
//
// Some callers cannot call cudaMalloc at all: engines whose device memory is
// one arena they own and hand out themselves, and plugins loaded into a host
// that forbids new device allocations after start-up (an allocation there
// can fail, or break the host's own accounting of device memory). For them
// this entry point runs the library's decode attention kernel (the same
// split-K kernel as slm_attend_cached_query) over a paged KV cache the caller
// owns, and keeps everything the kernel needs besides the caller's inputs and
// outputs (the step plan, split-K partials and merge counters, per-sequence
// status words, an error word) in one fixed file-scope device array below.
// Nothing is allocated per call.
//
// The array is kNoAllocScratchBytes (2 MiB). Every GPU that loads this
// library holds it until the process exits. It is shared by every call on
// that GPU and keeps the last call's contents; each call clears the parts
// that must start at zero (merge counters, status and error words). Calls
// whose work overlaps on the GPU (other streams, other host threads) race on
// it. A call waits for its stream before it returns.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "slmkv.h"
#include "slmkv_internal.h"
#include "slmkv_plan.h"

namespace slmkv {
void set_contextless_error(const std::string& message);  // slmkv_host.cpp
}

using namespace slmkv;

namespace {

// ---- fixed scratch layout ---------------------------------------------------
constexpr int kMaxPairs = 4096;                // (sequence, KV head) pairs per call
constexpr int kMaxChunks = 131072;             // stream blocks per call (16-token blocks x heads)
constexpr int kMaxSms = 160;                   // decode CTAs (one per SM)
constexpr int kMaxWarps = kMaxSms * kMaxDecodeWarps;  // decode warps: SMs x warps per CTA
constexpr int kMaxGroup = 8;                   // query heads per KV head
constexpr int kMaxSlots = 2 * kMaxSms;         // cross-CTA partials: < 2 per CTA

constexpr size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
constexpr size_t kOffPairs = 0;
constexpr size_t kOffChunks = align256(kOffPairs + sizeof(PairEntry) * kMaxPairs);
constexpr size_t kOffWarpStart = align256(kOffChunks + sizeof(int32_t) * kMaxChunks);
constexpr size_t kOffPartAcc = align256(kOffWarpStart + sizeof(int4) * 2 * kMaxWarps);
constexpr size_t kOffPartMl =
    align256(kOffPartAcc + sizeof(float) * kMaxSlots * kMaxGroup * kHeadDim);
constexpr size_t kOffCounters = align256(kOffPartMl + sizeof(float2) * kMaxSlots * kMaxGroup);
constexpr size_t kOffStatus = align256(kOffCounters + sizeof(int32_t) * kMaxPairs);
constexpr size_t kOffError = align256(kOffStatus + sizeof(int32_t) * kMaxPairs);
constexpr size_t kPlanBytes = kOffPartAcc;  // pairs + chunks + warp starts: uploaded per call
constexpr size_t kNoAllocScratchBytes = 2u << 20;
static_assert(kOffError + 256 <= kNoAllocScratchBytes, "scratch layout exceeds 2 MiB");

// The scratch itself. In host code this name is only a stand-in for the
// symbol; the device address comes from cudaGetSymbolAddress per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;  // guards the per-device set-up and the host staging below
void* g_scratch_dev[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};
// Host staging for the plan (filled, then copied to the scratch with one
// cudaMemcpyAsync from pageable memory, which returns once the source has
// been consumed); bounds[] is planner scratch.
alignas(16) unsigned char g_plan_host[kPlanBytes];
int32_t g_bounds[kMaxWarps + 1];
int32_t g_ctx_len[kMaxPairs];
int32_t g_status_host[kMaxPairs];  // sequences <= pairs
int32_t g_error_host;

slm_status fail(slm_status code, const char* fmt, ...) {
  char buf[400];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  set_contextless_error(buf);
  return code;
}

// Once per device, with that device current: the scratch's device address.
slm_status scratch_for_current_device(void** ptr, int* sms) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SLM_ERR_CUDA, "CUDA error in cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(SLM_ERR_CUDA, "device %d is outside the %d devices supported", dev, kMaxDevices);
  if (!g_scratch_dev[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(SLM_ERR_CUDA, "CUDA error in cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess)
      return fail(SLM_ERR_CUDA, "CUDA error in cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    g_sms[dev] = std::min(n, kMaxSms);
    g_scratch_dev[dev] = p;
  }
  *ptr = g_scratch_dev[dev];
  *sms = g_sms[dev];
  return SLM_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" slm_status slm_decode_attention_noalloc(
    const float* d_key_pool, const float* d_value_pool, int32_t num_blocks,
    int32_t num_query_heads, int32_t num_key_value_heads, const int32_t* h_block_table,
    int32_t max_blocks_per_sequence, const int32_t* h_lengths, int32_t n, const float* d_query,
    float* d_out, slm_stream stream) {
  const char* who = "slm_decode_attention_noalloc";
  if (!d_key_pool || !d_value_pool || !d_query || !d_out || !h_block_table || !h_lengths)
    return fail(SLM_ERR_INVALID_INPUT, "invalid input for %s: null pointer", who);
  if (!aligned16(d_key_pool) || !aligned16(d_value_pool) || !aligned16(d_query) ||
      !aligned16(d_out))
    return fail(SLM_ERR_INVALID_INPUT,
                "invalid input for %s: device buffers must be 16-byte aligned", who);
  if (num_blocks <= 0 || num_key_value_heads <= 0 || num_query_heads <= 0 ||
      num_query_heads % num_key_value_heads || max_blocks_per_sequence <= 0 || n <= 0)
    return fail(SLM_ERR_INVALID_INPUT, "invalid input for %s: dimensions must be positive and "
                "query heads a multiple of KV heads", who);
  const int32_t G = num_query_heads / num_key_value_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return fail(SLM_ERR_INVALID_INPUT,
                "invalid input for %s: query heads per KV head must be 1, 2, 4 or 8", who);
  // The plan names a chunk as block * kv_heads + head in an int32.
  if (static_cast<int64_t>(num_blocks) * num_key_value_heads > INT32_MAX)
    return fail(SLM_ERR_INVALID_INPUT,
                "invalid input for %s: %d blocks x %d KV heads exceed the int32 chunk index", who,
                num_blocks, num_key_value_heads);
  if (static_cast<int64_t>(n) * num_key_value_heads > kMaxPairs)
    return fail(SLM_ERR_INVALID_INPUT,
                "invalid input for %s: %lld (sequence, KV head) pairs exceed the %d its fixed "
                "scratch holds", who, static_cast<long long>(n) * num_key_value_heads, kMaxPairs);

  std::lock_guard<std::mutex> lock(g_mu);
  for (int32_t i = 0; i < n; ++i) {
    const int32_t L = h_lengths[i];
    if (L <= 0 || L > max_blocks_per_sequence * kBlockTokens)  // attention.rs:690-695
      return fail(SLM_ERR_INVALID_INPUT,
                  "invalid input for %s: sequence %d has length %d, outside 1..=%d", who, i, L,
                  max_blocks_per_sequence * kBlockTokens);
    const int32_t* row = h_block_table + static_cast<size_t>(i) * max_blocks_per_sequence;
    for (int32_t j = 0; j < (L + kBlockTokens - 1) / kBlockTokens; ++j)
      if (row[j] < 0 || row[j] >= num_blocks)
        return fail(SLM_ERR_INVALID_INPUT,
                    "invalid input for %s: sequence %d block %d is %d, outside 0..%d", who, i, j,
                    row[j], num_blocks);
    g_ctx_len[i] = L;
  }

  void* scratch = nullptr;
  int sms = 0;
  slm_status rc = scratch_for_current_device(&scratch, &sms);
  if (rc) return rc;
  const int32_t W = decode_warps(0, G);
  const PlanSizes sz = plan_sizes(n, g_ctx_len, num_key_value_heads, sms * W);
  if (sz.n_chunks > kMaxChunks)
    return fail(SLM_ERR_INVALID_INPUT,
                "invalid input for %s: %lld blocks to read exceed the %d its fixed scratch holds",
                who, static_cast<long long>(sz.n_chunks), kMaxChunks);

  auto* pairs = reinterpret_cast<PairEntry*>(g_plan_host + kOffPairs);
  auto* chunks = reinterpret_cast<int32_t*>(g_plan_host + kOffChunks);
  auto* wstart = reinterpret_cast<int4*>(g_plan_host + kOffWarpStart);
  const int32_t slots = build_decode_plan(
      n, g_ctx_len,
      [&](int32_t i, int32_t j) {
        return h_block_table[static_cast<size_t>(i) * max_blocks_per_sequence + j];
      },
      num_key_value_heads, W, sz, pairs, chunks, wstart, g_bounds);
  if (slots > kMaxSlots)  // fewer than two per decode CTA by construction
    return fail(SLM_ERR_INVALID_INPUT, "invalid input for %s: plan needs %d merge slots", who, slots);

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned char* dev = static_cast<unsigned char*>(scratch);
  cudaError_t e = cudaSuccess;
  // Plan: pairs, chunk stream and warp starts (only the used prefix of each).
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(dev + kOffPairs, pairs, sizeof(PairEntry) * sz.n_pairs,
                        cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(dev + kOffChunks, chunks, sizeof(int32_t) * sz.n_chunks,
                        cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(dev + kOffWarpStart, wstart, sizeof(int4) * 2 * sz.n_warps,
                        cudaMemcpyHostToDevice, s);
  // What must start at zero: the merge counters, the status words and the
  // error word.
  if (e == cudaSuccess)
    e = cudaMemsetAsync(dev + kOffCounters, 0, sizeof(int32_t) * sz.n_pairs, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(dev + kOffStatus, 0, sizeof(int32_t) * n, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(dev + kOffError, 0, sizeof(int32_t), s);
  if (e != cudaSuccess)
    return fail(SLM_ERR_CUDA, "CUDA error in %s (plan upload): %s", who, cudaGetErrorString(e));

  StreamDecodeLaunch p{};
  p.g.k = const_cast<float*>(d_key_pool);
  p.g.v = const_cast<float*>(d_value_pool);
  p.g.layer_elems = static_cast<int64_t>(num_blocks) * num_key_value_heads * kBlockTokens * kHeadDim;
  p.g.block_table = nullptr;  // the plan carries the physical blocks
  p.g.max_blocks_per_seq = max_blocks_per_sequence;
  p.g.num_blocks = num_blocks;
  p.g.num_layers = 1;
  p.g.kv_heads = num_key_value_heads;
  p.g.q_heads = num_query_heads;
  p.g.bf16 = 0;
  p.g.rope = nullptr;  // attention only: the query arrives rotated
  p.g.context_length = max_blocks_per_sequence * kBlockTokens;
  p.g.error = reinterpret_cast<int32_t*>(dev + kOffError);
  p.layer = 0;
  p.n_layers = 1;
  p.pairs = reinterpret_cast<const PairEntry*>(dev + kOffPairs);
  p.n_pairs = static_cast<int32_t>(sz.n_pairs);
  p.chunks = reinterpret_cast<const int32_t*>(dev + kOffChunks);
  p.total_blocks = static_cast<int32_t>(sz.n_chunks);
  p.warp_start = reinterpret_cast<const int4*>(dev + kOffWarpStart);
  p.n_warps = sz.n_warps;
  p.q[0] = d_query;
  p.out[0] = d_out;
  p.part_acc = reinterpret_cast<float*>(dev + kOffPartAcc);
  p.part_ml = reinterpret_cast<float2*>(dev + kOffPartMl);
  p.counters = reinterpret_cast<int32_t*>(dev + kOffCounters);
  p.status = reinterpret_cast<int32_t*>(dev + kOffStatus);
  p.fused = 0;
  e = launch_decode(p, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(&g_error_host, dev + kOffError, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(g_status_host, dev + kOffStatus, sizeof(int32_t) * n,
                        cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess)
    return fail(SLM_ERR_CUDA, "CUDA error in %s: %s", who, cudaGetErrorString(e));
  if (g_error_host & kErrTimeout)
    return fail(SLM_ERR_DEVICE_TIMEOUT, "%s: a device wait timed out", who);
  if (g_error_host)
    return fail(SLM_ERR_INVALID_INPUT, "invalid input for %s: out-of-pool block id", who);
  for (int32_t i = 0; i < n; ++i)
    if (g_status_host[i] & kStatusNonFiniteScore)  // softmax.rs:17-22
      return fail(SLM_ERR_NON_FINITE,
                  "invalid input for softmax: all input values must be finite (sequence %d)", i);
  return SLM_OK;
}
