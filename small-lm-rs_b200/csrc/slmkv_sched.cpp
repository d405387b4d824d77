// Continuous-batching scheduler over one context's sequences (C ABI in
// include/slmkv.h). Host bookkeeping only: it decides which requests run in a
// step and how many of their tokens; the caller runs the KV batches. The
// reference serves one request at a time (rust/server/src/worker.rs:87-98):
// GenerationService prefills the prompt, picks the first token from the last
// prompt position, then decodes one token per step until max_new_tokens.
// Here many requests do that together.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <deque>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "slmkv.h"

namespace {

constexpr int32_t kBlock = 16;
int32_t blocks_for(int32_t tokens) { return (tokens + kBlock - 1) / kBlock; }

struct Request {
  int64_t id = 0;
  int32_t prompt_len = 0, max_new = 0;
  int32_t seq = -1;           // sequence slot while admitted
  int32_t cached = 0;         // positions in the KV cache
  int32_t target = 0;         // positions to prefill before decoding
  int32_t generated = 0;      // output tokens produced
  bool first_from_prefill = true;  // the prompt's end yields the first token
  uint64_t order = 0;         // admission order
};

}  // namespace

struct slm_sched {
  slm_ctx* ctx = nullptr;
  slm_sched_config cfg{};
  int32_t num_blocks = 0, context_length = 0;
  std::deque<std::unique_ptr<Request>> waiting;   // preempted ones go to the front
  std::vector<std::unique_ptr<Request>> running;  // in admission order
  std::unordered_map<int64_t, bool> known;        // submitted and not finished
  uint64_t next_order = 0;
  int64_t preemptions = 0, generated_tokens = 0;
  // the last plan
  bool planned = false;
  std::vector<Request*> plan_decode, plan_prefill;
  std::vector<int32_t> plan_count;
};

namespace {

int32_t held_blocks(const slm_sched* s) {
  int32_t n = 0;
  for (const auto& r : s->running) n += blocks_for(r->cached);
  return n;
}

// Frees the newest running request's sequence and puts it back at the front
// of the queue, to prefill what it had cached again: its prompt and the
// tokens it generated (a request preempted inside its prompt keeps the
// whole prompt as its target).
void preempt_newest(slm_sched* s) {
  std::unique_ptr<Request> r = std::move(s->running.back());
  s->running.pop_back();
  slm_seq_free(s->ctx, r->seq);
  r->seq = -1;
  r->target = std::max(r->target, r->cached);
  r->cached = 0;
  r->first_from_prefill = (r->generated == 0);
  s->waiting.push_front(std::move(r));
  ++s->preemptions;
}

}  // namespace

extern "C" {

slm_status slm_sched_create(slm_ctx* ctx, const slm_sched_config* config, slm_sched** out) {
  if (!ctx || !config || !out || config->max_running < 1 || config->max_prefill_tokens < 1)
    return SLM_ERR_INVALID_INPUT;
  slm_config c{};
  slm_status rc = slm_ctx_config(ctx, &c);
  if (rc) return rc;
  auto s = std::make_unique<slm_sched>();
  s->ctx = ctx;
  s->cfg = *config;
  s->cfg.max_running = std::min(config->max_running, c.max_sequences);
  s->num_blocks = c.num_blocks;
  s->context_length = c.context_length;
  *out = s.release();
  return SLM_OK;
}

slm_status slm_sched_destroy(slm_sched* s) {
  if (!s) return SLM_ERR_INVALID_INPUT;
  for (auto& r : s->running) slm_seq_free(s->ctx, r->seq);
  delete s;
  return SLM_OK;
}

slm_status slm_sched_submit(slm_sched* s, int64_t request_id, int32_t prompt_len,
                            int32_t max_new_tokens) {
  if (!s) return SLM_ERR_INVALID_INPUT;
  if (prompt_len < 1 || max_new_tokens < 1)
    return SLM_ERR_INVALID_INPUT;
  // kv_cache.rs:203-211: the request must fit its sequence capacity.
  if (static_cast<int64_t>(prompt_len) + max_new_tokens > s->context_length)
    return SLM_ERR_CAPACITY;
  if (blocks_for(prompt_len + max_new_tokens) > s->num_blocks) return SLM_ERR_POOL_EXHAUSTED;
  if (s->known.count(request_id)) return SLM_ERR_INVALID_INPUT;
  auto r = std::make_unique<Request>();
  r->id = request_id;
  r->prompt_len = prompt_len;
  r->max_new = max_new_tokens;
  r->target = prompt_len;
  s->known[request_id] = true;
  s->waiting.push_back(std::move(r));
  return SLM_OK;
}

slm_status slm_sched_plan(slm_sched* s, int32_t* n_decode, int32_t* decode_seq,
                          int32_t* n_prefill, int32_t* prefill_seq, int32_t* prefill_count) {
  if (!s || !n_decode || !n_prefill || !decode_seq || !prefill_seq || !prefill_count)
    return SLM_ERR_INVALID_INPUT;
  bool admit = true;  // no admission after a preemption in the same plan
  for (;;) {
    // Admission, in arrival order, while the pool holds the prompt.
    int32_t free_blocks = s->num_blocks - held_blocks(s);
    while (admit && !s->waiting.empty() &&
           static_cast<int32_t>(s->running.size()) < s->cfg.max_running) {
      Request* r = s->waiting.front().get();
      if (blocks_for(r->target) > free_blocks) break;
      int32_t seq = -1;
      if (slm_seq_create(s->ctx, std::min(s->context_length, r->prompt_len + r->max_new), &seq))
        break;  // no sequence slot
      r->seq = seq;
      r->order = s->next_order++;
      free_blocks -= blocks_for(r->target);  // kept aside for its prompt
      s->running.push_back(std::move(s->waiting.front()));
      s->waiting.pop_front();
    }
    // The step: decode tokens for cached prompts, prompt chunks for the rest.
    s->plan_decode.clear();
    s->plan_prefill.clear();
    s->plan_count.clear();
    int32_t budget = s->cfg.max_prefill_tokens;
    int32_t need = 0;  // blocks the step adds
    for (auto& up : s->running) {
      Request* r = up.get();
      if (r->cached >= r->target) {
        s->plan_decode.push_back(r);
        need += blocks_for(r->cached + 1) - blocks_for(r->cached);
      } else if (budget > 0) {
        const int32_t t = std::min(budget, r->target - r->cached);
        budget -= t;
        s->plan_prefill.push_back(r);
        s->plan_count.push_back(t);
        need += blocks_for(r->cached + t) - blocks_for(r->cached);
      }
    }
    if (need <= s->num_blocks - held_blocks(s) || s->running.size() <= 1) break;
    preempt_newest(s);  // the pool cannot hold the step: recompute the newest later
    admit = false;
  }
  *n_decode = static_cast<int32_t>(s->plan_decode.size());
  for (size_t i = 0; i < s->plan_decode.size(); ++i) decode_seq[i] = s->plan_decode[i]->seq;
  *n_prefill = static_cast<int32_t>(s->plan_prefill.size());
  for (size_t i = 0; i < s->plan_prefill.size(); ++i) {
    prefill_seq[i] = s->plan_prefill[i]->seq;
    prefill_count[i] = s->plan_count[i];
  }
  s->planned = true;
  return SLM_OK;
}

slm_status slm_sched_plan_requests(const slm_sched* s, int64_t* decode_request, int32_t* decode_pos,
                                   int64_t* prefill_request, int32_t* prefill_pos) {
  if (!s || !s->planned) return SLM_ERR_INVALID_INPUT;
  for (size_t i = 0; i < s->plan_decode.size(); ++i) {
    if (decode_request) decode_request[i] = s->plan_decode[i]->id;
    if (decode_pos) decode_pos[i] = s->plan_decode[i]->cached;
  }
  for (size_t i = 0; i < s->plan_prefill.size(); ++i) {
    if (prefill_request) prefill_request[i] = s->plan_prefill[i]->id;
    if (prefill_pos) prefill_pos[i] = s->plan_prefill[i]->cached;
  }
  return SLM_OK;
}

slm_status slm_sched_commit(slm_sched* s, const int32_t* decode_status,
                            const int32_t* prefill_status, int32_t* n_finished,
                            int64_t* finished_id, int32_t* finished_status, int32_t* h_generated) {
  if (!s || !n_finished || !finished_id || !finished_status) return SLM_ERR_INVALID_INPUT;
  if (!s->planned) return SLM_ERR_INVALID_INPUT;
  if ((!s->plan_decode.empty() && !decode_status) || (!s->plan_prefill.empty() && !prefill_status))
    return SLM_ERR_INVALID_INPUT;
  std::unordered_map<Request*, int32_t> failed;
  for (size_t i = 0; i < s->plan_decode.size(); ++i) {
    Request* r = s->plan_decode[i];
    if (decode_status[i] != SLM_OK) {
      failed[r] = decode_status[i];
      continue;
    }
    r->cached += 1;
    r->generated += 1;
    ++s->generated_tokens;
  }
  for (size_t i = 0; i < s->plan_prefill.size(); ++i) {
    Request* r = s->plan_prefill[i];
    if (prefill_status[i] != SLM_OK) {
      failed[r] = prefill_status[i];
      continue;
    }
    r->cached += s->plan_count[i];
    if (r->cached == r->target && r->first_from_prefill) {
      r->generated = 1;  // the first token, from the prompt's last position
      r->first_from_prefill = false;
      ++s->generated_tokens;
    }
  }
  int32_t nf = 0;
  std::vector<std::unique_ptr<Request>> keep;
  keep.reserve(s->running.size());
  for (auto& up : s->running) {
    Request* r = up.get();
    auto f = failed.find(r);
    const bool done = (f != failed.end()) || r->generated >= r->max_new;
    if (!done) {
      keep.push_back(std::move(up));
      continue;
    }
    finished_id[nf] = r->id;
    finished_status[nf] = (f != failed.end()) ? f->second : SLM_OK;
    if (h_generated) h_generated[nf] = r->generated;
    ++nf;
    slm_seq_free(s->ctx, r->seq);
    s->known.erase(r->id);
  }
  s->running.swap(keep);
  *n_finished = nf;
  s->planned = false;
  return SLM_OK;
}

slm_status slm_sched_counts(const slm_sched* s, int32_t* waiting, int32_t* running,
                            int64_t* preemptions, int64_t* generated_tokens) {
  if (!s) return SLM_ERR_INVALID_INPUT;
  if (waiting) *waiting = static_cast<int32_t>(s->waiting.size());
  if (running) *running = static_cast<int32_t>(s->running.size());
  if (preemptions) *preemptions = s->preemptions;
  if (generated_tokens) *generated_tokens = s->generated_tokens;
  return SLM_OK;
}

}  // extern "C"
