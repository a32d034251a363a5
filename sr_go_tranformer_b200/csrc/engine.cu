// engine.cu -- host-side restatement of the reference's Engine actor
// (cmd/monolith/monolith.go:7629-8476, "M:line") over the device step.
//
// The Go engine keeps its own loop and calls sr_step / sr_sample through cgo;
// this C++ engine reproduces that loop's integer decisions (admission, page
// reservation, scheduleTokens, the LIFO page pool, finishing) for callers that
// have no Go runtime (tests, benchmarks), including the one-entry prefix
// snapshot (M:5868-5952) whose page copies run on the device.  HTTP, SSE
// streaming, tokenisation and cancellation watchers are outside this
// restatement.
#include <algorithm>
#include <chrono>
#include <cstring>
#include <deque>
#include <string>
#include <vector>

#include "../../include/srstep.h"
#include "srstep_internal.h"

namespace {

using Clock = std::chrono::steady_clock;

struct EngRequest {
  int64_t id;
  std::vector<int32_t> ids;
  int32_t max_tokens;
  sr_sampling s;
  uint64_t seed;
  Clock::time_point started;  // Request.Started (submit time)
};

struct EngSession {
  EngRequest req;
  std::vector<int32_t> pages;  // KVCache.Pages (page ids)
  int32_t reserved = 0;        // KVCache.reserved
  bool shared = false;         // KVCache.shared != nil (the engine has one snapshot)
  int32_t shared_pages = 0;    // KVCache.sharedPages
  int64_t prefix_epoch = 0;    // engineSession.PrefixEpoch
  int32_t pos = 0;             // KVCache.Pos
  int32_t cursor = 0;          // engineSession.Cursor
  std::vector<int32_t> output, history;
  uint64_t rng = 0;            // engineSession.RNG
  Clock::time_point last_token;  // engineSession.LastToken
  bool has_token = false;
  sr_text_decoder* text = nullptr;  // engineSession.Text (token events only)
};

// TokenEvent (M:7643-7647): one sampled token and the text it completes.
struct TextEvent {
  int64_t request_id;
  int32_t token_id;
  std::string text;
  int32_t final;
};

struct Finished {
  int64_t id;
  std::vector<int32_t> out;
  int32_t reason;  // 0 length, 1 eos, 2 error, 3 busy
};

// prefixSnapshot (M:5868-5877).  Its i-th page is device page limit + i of the
// engine's pool; the pool holds prefix_limit such pages after the Limit pages
// that pagePool hands out.  valid stands for p.model != nil (one model per
// engine, whose revision never changes).
struct PrefixSnapshot {
  bool valid = false;
  std::vector<int32_t> ids;
  int32_t pages = 0;  // len(p.pages)
  int32_t borrowers = 0;
  bool include_tail = false;
};

}  // namespace

struct sr_engine {
  sr_model* m = nullptr;
  sr_kvpool* pool = nullptr;
  sr_engine_config c;
  // pagePool (M:5849-5866): Limit, Reserved, Allocated and the LIFO free list.
  int64_t limit = 0, reserved = 0, allocated = 0;
  std::vector<int32_t> free_pages;
  PrefixSnapshot prefix;
  int64_t prefix_limit = 0, prefix_epoch = 0;
  bool clear_pending = false;
  std::deque<EngRequest> queue;
  std::vector<EngSession> sessions;
  int32_t rotation = 0;
  int64_t next_id = 0;
  std::deque<Finished> finished;
  // Token events (M:8451-8462): the pieces table (bytes of every id) and the
  // decoder flags newTextDecoder would pick; off until sr_engine_set_pieces.
  bool text_on = false;
  int32_t text_flags = 0;
  std::string pieces;
  std::vector<int64_t> piece_off;
  std::vector<uint8_t> fallback;
  std::deque<TextEvent> events;
  sr_engine_stats st{};
  std::vector<int32_t> last_counts;
  // firstTokenLatency / tokenGap observations (M:8441-8447), in seconds
  std::vector<double> ttft, itl;
  // per-tick scratch
  std::vector<int32_t> pos, toff, tokens, poff, pids, counts, hoff, hist, ids_out;
  std::vector<uint8_t> want;
  std::vector<sr_sampling> settings;
  std::vector<uint64_t> rng;
};

// pagePool.acquire (M:5854-5866): pop the tail of the free list, else allocate.
static int32_t acquire(sr_engine* e) {
  if (!e->free_pages.empty()) {
    int32_t p = e->free_pages.back();
    e->free_pages.pop_back();
    return p;
  }
  return (int32_t)(e->allocated++);
}

// KVCache.Close (M:6044-6062): owned pages return to the free list in page
// order; borrowed snapshot pages only drop the borrow.
static void close_session(sr_engine* e, EngSession& s) {
  e->free_pages.insert(e->free_pages.end(), s.pages.begin() + s.shared_pages, s.pages.end());
  e->reserved -= s.reserved;
  if (s.shared) {
    PrefixSnapshot& p = e->prefix;
    p.borrowers--;
    if (p.borrowers == 0 && !p.valid) p.pages = 0;
    s.shared = false;
  }
  s.pages.clear();
  s.shared_pages = 0;
  if (s.text) {
    sr_text_decoder_destroy(s.text);
    s.text = nullptr;
  }
}

static int32_t snapshot_page(const sr_engine* e, int32_t i) { return (int32_t)(e->limit + i); }

// prefixSnapshot.restore (M:5881-5905): borrow the snapshot's whole matching
// pages; with tail reuse, copy the matching rows of the next page into a page
// of the session's own.  The last prompt id always runs through the model.
static int restore_prefix(sr_engine* e, EngSession& s) {
  PrefixSnapshot& p = e->prefix;
  const std::vector<int32_t>& ids = s.req.ids;
  if (!p.valid || ids.size() < 2) return SR_OK;
  const size_t n = std::min(p.ids.size(), ids.size() - 1);
  size_t matched = 0;
  while (matched < n && p.ids[matched] == ids[matched]) matched++;
  const int32_t pt = e->m->d.page_tokens;
  const int32_t full = (int32_t)(matched / pt);
  if (full > 0) {
    for (int32_t i = 0; i < full; i++) s.pages.push_back(snapshot_page(e, i));
    s.shared = true;
    s.shared_pages = full;
    p.borrowers++;
  }
  s.pos = full * pt;
  const int32_t tail = (int32_t)(matched % pt);
  if (p.include_tail && tail > 0) {
    while ((int64_t)s.pages.size() < full + 1) s.pages.push_back(acquire(e));  // ensurePages(matched)
    int rc = sr_kvpool_copy_rows(e->pool, s.pages[full], snapshot_page(e, full), tail);
    if (rc != SR_OK) return rc;
    s.pos = (int32_t)matched;
  }
  return SR_OK;
}

// prefixSnapshot.capture (M:5927-5952): keep the committed positions of a
// successfully finished session.  Skipped while another session borrows the
// snapshot; the session's own borrowed pages are already in place.
static int capture_prefix(sr_engine* e, const EngSession& s) {
  PrefixSnapshot& p = e->prefix;
  const bool sole = s.shared && p.borrowers == 1 && p.valid;
  if (p.borrowers != 0 && !sole) return SR_OK;
  const int64_t pt = e->m->d.page_tokens;
  int64_t positions = s.pos;
  if (!p.include_tail) positions -= positions % pt;
  const int64_t n = std::min<int64_t>(e->prefix_limit, (positions + pt - 1) / pt);
  positions = std::min<int64_t>(positions, n * pt);
  if (n == 0) return SR_OK;
  if (p.pages < n) p.pages = (int32_t)n;
  for (int64_t i = 0; i < n; i++) {
    const int32_t dst = snapshot_page(e, (int32_t)i);
    if (dst != s.pages[i]) {
      int rc = sr_kvpool_copy_rows(e->pool, dst, s.pages[i], (int32_t)std::min<int64_t>(pt, positions - i * pt));
      if (rc != SR_OK) return rc;
    }
  }
  p.ids.assign(s.history.begin(), s.history.begin() + positions);
  p.valid = true;
  return SR_OK;
}

// prefixSnapshot.clear (M:5915-5921) behind the actor's clearPrefix (M:8236-8241).
static void clear_prefix(sr_engine* e) {
  e->prefix_epoch++;
  e->prefix.ids.clear();
  e->prefix.valid = false;
  if (e->prefix.borrowers == 0) e->prefix.pages = 0;
  e->clear_pending = false;
}

static void account(sr_engine* e) {  // the actor's accounting (M:8230-8235)
  e->st.prefix_bytes = (int64_t)e->prefix.pages * e->m->dm.page_elems * 4;
  e->st.pool_reserved = e->reserved;
  e->st.pool_allocated = e->allocated + e->prefix.pages;
}

static void finish(sr_engine* e, EngSession& s, int32_t reason) {
  // finish (M:8285-8293): a successful session whose epoch is current offers its
  // positions to the snapshot before its cache closes.
  if (reason <= 1 && s.prefix_epoch == e->prefix_epoch && e->prefix_limit > 0) {
    int rc = capture_prefix(e, s);
    if (rc != SR_OK) reason = 2;
  }
  close_session(e, s);
  e->st.active--;
  if (reason <= 1) e->st.completed++;
  else e->st.failed++;
  e->finished.push_back(Finished{s.req.id, s.output, reason});
}

// scheduleTokens (M:8180-8210).
static int32_t schedule_tokens(const std::vector<EngSession>& ss, std::vector<int32_t>& counts, int32_t budget,
                               int32_t chunk, int32_t mixed_chunk, int32_t start) {
  const int32_t n = (int32_t)ss.size();
  for (const auto& s : ss)
    if (s.cursor == (int32_t)s.req.ids.size()) {
      chunk = std::min(chunk, mixed_chunk);
      break;
    }
  int32_t total = n;
  counts.assign(n, 1);
  while (total < budget) {
    bool progress = false;
    for (int32_t j = 0; j < n; j++) {
      int32_t i = (start + j) % n;
      int32_t remaining = (int32_t)ss[i].req.ids.size() - ss[i].cursor;
      if (counts[i] < std::min(chunk, remaining)) {
        counts[i]++;
        total++;
        progress = true;
        if (total == budget) break;
      }
    }
    if (!progress) break;
  }
  return total;
}

extern "C" int sr_engine_create(sr_model* m, const sr_engine_config* cfg, sr_engine** out) {
  if (!m || !cfg || !out) return sr_fail(SR_EINVAL, "null argument");
  *out = nullptr;
  sr_engine_config c = *cfg;
  // normalizeEngineConfig (M:7983-8012).
  if (c.prefill_chunk == 0) c.prefill_chunk = 16;
  if (c.mixed_prefill_chunk == 0) c.mixed_prefill_chunk = 1;
  if (c.token_budget == 0) c.token_budget = std::max(c.max_batch, 64);
  if (c.max_batch < 1 || c.max_batch > 256 || c.cache_bytes < 1 || c.prefill_chunk < 1 || c.prefill_chunk > 1024 ||
      c.mixed_prefill_chunk < 1 || c.mixed_prefill_chunk > 1024 || c.token_budget < c.max_batch ||
      c.token_budget > 1024)
    return sr_fail(SR_EINVAL, "invalid engine capacity or token budget");
  if (c.prefix_cache_bytes < 0 || c.prefix_cache_bytes >= c.cache_bytes)  // M:7999-8003
    return sr_fail(SR_EINVAL, "prefix cache must be nonnegative and smaller than total KV budget");
  if (c.prefix_cache_tail && c.prefix_cache_bytes == 0)
    return sr_fail(SR_EINVAL, "prefix cache tail reuse requires a positive prefix cache budget");
  const int64_t page_bytes = m->dm.page_elems * 4;
  const int64_t prefix_limit = c.prefix_cache_bytes / page_bytes;  // newEngine (M:8031-8035)
  if (c.prefix_cache_bytes != 0 && prefix_limit == 0)
    return sr_fail(SR_EINVAL, "prefix cache budget cannot hold one KV page");
  const int64_t limit = (c.cache_bytes - c.prefix_cache_bytes) / page_bytes;
  if (limit < 1) return sr_fail(SR_EINVAL, "cache budget cannot hold one KV page");
  sr_engine* e = new sr_engine();
  e->m = m;
  e->c = c;
  e->limit = limit;
  e->prefix_limit = prefix_limit;
  e->prefix.include_tail = c.prefix_cache_tail != 0;
  int rc = sr_kvpool_create(m, limit + prefix_limit, &e->pool);
  if (rc != SR_OK) {
    delete e;
    return rc;
  }
  e->st.pool_limit = limit;
  *out = e;
  return SR_OK;
}

extern "C" int sr_engine_destroy(sr_engine* e) {
  if (!e) return sr_fail(SR_EINVAL, "null engine");
  for (auto& s : e->sessions)
    if (s.text) sr_text_decoder_destroy(s.text);
  if (e->pool) sr_kvpool_destroy(e->pool);
  delete e;
  return SR_OK;
}

extern "C" int sr_engine_submit(sr_engine* e, const sr_request* r, int64_t* request_id) {
  if (!e || !r || !request_id) return sr_fail(SR_EINVAL, "null argument");
  if (r->n_ids < 1 || !r->ids) return sr_fail(SR_EINVAL, "empty prompt");
  const sr_model_desc& d = e->m->d;
  // prepareInput's bounds (M:7466-7497): ids in vocabulary, prompt+max_tokens <= context.
  if (r->max_tokens < 1 || r->max_tokens > d.context || (int64_t)r->n_ids + r->max_tokens > d.context)
    return sr_fail(SR_EINVAL, "prompt plus max_tokens exceeds the model context");
  for (int32_t i = 0; i < r->n_ids; i++)
    if (r->ids[i] < 0 || r->ids[i] >= d.vocab) return sr_fail(SR_EINVAL, "token outside vocabulary");
  const int64_t pt = d.page_tokens;
  const int64_t pages = ((int64_t)r->n_ids + r->max_tokens + pt - 1) / pt;
  if (pages > e->limit) return sr_fail(SR_EINVAL, "request exceeds total KV cache budget");  // M:8097-8100
  EngRequest q;
  q.id = e->next_id++;
  q.ids.assign(r->ids, r->ids + r->n_ids);
  q.max_tokens = r->max_tokens;
  q.s = r->sampling;
  q.seed = r->seed;
  q.started = Clock::now();
  e->queue.push_back(std::move(q));
  e->st.submitted++;
  *request_id = e->next_id - 1;
  return SR_OK;
}

extern "C" int sr_engine_tick(sr_engine* e, int32_t* rows) {
  if (!e || !rows) return sr_fail(SR_EINVAL, "null argument");
  *rows = 0;
  const int64_t pt = e->m->d.page_tokens;
  if (e->clear_pending && e->sessions.empty()) clear_prefix(e);
  // Admission (M:8325-8366): reserve whole pages for prompt + max_tokens, then
  // restore the matching prefix from the snapshot.
  while ((int)e->sessions.size() < e->c.max_batch && !e->queue.empty()) {
    EngRequest r = std::move(e->queue.front());
    e->queue.pop_front();
    const int64_t pages = ((int64_t)r.ids.size() + r.max_tokens + pt - 1) / pt;
    if (e->reserved + pages > e->limit) {
      e->st.rejected++;
      e->finished.push_back(Finished{r.id, {}, 3});
      continue;
    }
    EngSession s;
    s.reserved = (int32_t)pages;
    e->reserved += pages;
    s.history = r.ids;
    s.rng = r.seed;  // RNG{r.Sampling.Seed}
    s.req = std::move(r);
    s.prefix_epoch = e->prefix_epoch;
    int rc = restore_prefix(e, s);
    if (rc != SR_OK) {
      std::string msg = sr_last_error();
      close_session(e, s);
      e->st.failed++;
      e->finished.push_back(Finished{s.req.id, {}, 2});
      account(e);
      sr_fail(rc, msg);
      return rc;
    }
    if (s.pos > 0) {
      e->st.prefix_hits++;
      e->st.prefix_tokens += s.pos;
    }
    s.cursor = s.pos;  // engineSession.Cursor = cache.Pos
    if (e->text_on) {  // newTextDecoder (M:8363)
      rc = sr_text_decoder_create(e->text_flags, e->fallback.empty() ? nullptr : e->fallback.data(),
                                  (int32_t)e->fallback.size(), &s.text);
      if (rc != SR_OK) {  // the request fails as a whole, like a failed prefix restore
        std::string msg = sr_last_error();
        close_session(e, s);
        e->st.failed++;
        e->finished.push_back(Finished{s.req.id, {}, 2});
        account(e);
        sr_fail(rc, msg);
        return rc;
      }
    }
    e->sessions.push_back(std::move(s));
    e->st.active++;
    account(e);
  }
  e->st.queued = (int64_t)e->queue.size();
  if (e->sessions.empty()) return SR_OK;
  const int32_t n = (int32_t)e->sessions.size();
  const int32_t total = schedule_tokens(e->sessions, e->counts, e->c.token_budget, e->c.prefill_chunk,
                                        e->c.mixed_prefill_chunk, e->rotation % n);
  e->rotation = (e->rotation + 1) % n;
  e->last_counts = e->counts;
  // Build the ragged batch: chunks, wantLogits, lazily acquired pages (M:8372-8381, 6362-6364).
  e->pos.assign(n, 0);
  e->toff.assign(n + 1, 0);
  e->poff.assign(n + 1, 0);
  e->want.assign(n, 0);
  e->tokens.clear();
  e->pids.clear();
  e->hoff.assign(n + 1, 0);
  e->hist.clear();
  e->settings.resize(n);
  e->rng.resize(n);
  e->ids_out.assign(n, -1);
  for (int32_t i = 0; i < n; i++) {
    EngSession& s = e->sessions[i];
    const int32_t plen = (int32_t)s.req.ids.size();
    e->want[i] = (s.cursor + e->counts[i] >= plen) ? 1 : 0;
    if (s.cursor < plen)
      e->tokens.insert(e->tokens.end(), s.req.ids.begin() + s.cursor, s.req.ids.begin() + s.cursor + e->counts[i]);
    else
      e->tokens.push_back(s.output.back());
    e->toff[i + 1] = (int32_t)e->tokens.size();
    const int32_t len = e->toff[i + 1] - e->toff[i];
    const int64_t needed = ((int64_t)s.pos + len + pt - 1) / pt;  // ensurePages (M:6023-6037)
    while ((int64_t)s.pages.size() < needed) s.pages.push_back(acquire(e));
    e->pos[i] = s.pos;
    e->pids.insert(e->pids.end(), s.pages.begin(), s.pages.end());
    e->poff[i + 1] = (int32_t)e->pids.size();
    if (e->want[i]) e->hist.insert(e->hist.end(), s.history.begin(), s.history.end());
    e->hoff[i + 1] = (int32_t)e->hist.size();
    e->settings[i] = s.req.s;
    e->rng[i] = s.rng;
  }
  sr_batch b;
  b.n_sessions = n;
  b.pos = e->pos.data();
  b.token_offsets = e->toff.data();
  b.tokens = e->tokens.data();
  b.page_offsets = e->poff.data();
  b.page_ids = e->pids.data();
  b.want_logits = e->want.data();
  *rows = total;
  e->st.ticks++;
  e->st.peak_tick_tokens = std::max<int64_t>(e->st.peak_tick_tokens, total);
  int rc = sr_step_sample(e->m, e->pool, &b, e->settings.data(), e->hoff.data(), e->hist.data(), e->rng.data(),
                          e->c.blocked_id, e->ids_out.data());
  if (rc != SR_OK) {
    // A failed step finishes every active session with the error (M:8409-8418).
    std::string msg = sr_last_error();
    for (auto& s : e->sessions) finish(e, s, 2);
    e->sessions.clear();
    account(e);
    sr_fail(rc, msg);
    return rc;
  }
  // Commit positions (M:6452-6454), advance cursors, sample, finish (M:8419-8474).
  std::vector<EngSession> alive;
  alive.reserve(n);
  for (int32_t i = 0; i < n; i++) {
    EngSession& s = e->sessions[i];
    s.pos += e->toff[i + 1] - e->toff[i];
    const int32_t plen = (int32_t)s.req.ids.size();
    if (s.cursor < plen) {
      s.cursor += e->counts[i];
      e->st.input_tokens += e->counts[i];
    }
    if (s.cursor < plen) {
      alive.push_back(std::move(s));
      continue;
    }
    const int32_t id = e->ids_out[i];
    s.rng = e->rng[i];
    const Clock::time_point now = Clock::now();  // after the step's synchronising sample call
    if (!s.has_token) e->ttft.push_back(std::chrono::duration<double>(now - s.req.started).count());
    else e->itl.push_back(std::chrono::duration<double>(now - s.last_token).count());
    s.last_token = now;
    s.has_token = true;
    e->st.generated_tokens++;
    s.output.push_back(id);
    s.history.push_back(id);
    int32_t reason = -1;
    if (e->c.eos_id >= 0 && id == e->c.eos_id) reason = 1;
    else if ((int32_t)s.output.size() == s.req.max_tokens) reason = 0;
    if (s.text) {  // TokenEvent{id, Text.PushToken(id, pieces[id], final)} (M:8458-8459)
      const bool in_vocab = id >= 0 && (size_t)id + 1 < e->piece_off.size();
      const int64_t lo = in_vocab ? e->piece_off[id] : 0, len = in_vocab ? e->piece_off[id + 1] - lo : 0;
      std::string out((size_t)(3 * len + 4096), '\0');
      int64_t n_out = 0, queued = 0;
      sr_text_decoder_push_token(s.text, id, (const uint8_t*)e->pieces.data() + lo, len, reason >= 0, &out[0],
                                 (int64_t)out.size(), &n_out, &queued);
      out.resize((size_t)n_out);
      while (queued > 0) {
        std::string more((size_t)queued + 16, '\0');
        int64_t m = 0;
        sr_text_decoder_push(s.text, nullptr, 0, 0, &more[0], (int64_t)more.size(), &m, &queued);
        out.append(more, 0, (size_t)m);
      }
      e->events.push_back(TextEvent{s.req.id, id, std::move(out), reason >= 0 ? 1 : 0});
    }
    if (reason >= 0) finish(e, s, reason);
    else alive.push_back(std::move(s));
  }
  e->sessions = std::move(alive);
  account(e);
  return SR_OK;
}

extern "C" int sr_engine_clear_prefix(sr_engine* e) {
  if (!e) return sr_fail(SR_EINVAL, "null engine");
  e->clear_pending = true;
  if (e->sessions.empty()) clear_prefix(e);
  account(e);
  return SR_OK;
}

extern "C" int sr_engine_poll(sr_engine* e, int64_t* request_id, int32_t* out_ids, int32_t cap, int32_t* n_out,
                              int32_t* reason) {
  if (!e || !request_id || !n_out || !reason) return sr_fail(SR_EINVAL, "null argument");
  if (e->finished.empty()) {
    *request_id = -1;
    *n_out = 0;
    *reason = -1;
    return SR_OK;
  }
  Finished f = std::move(e->finished.front());
  e->finished.pop_front();
  *request_id = f.id;
  *reason = f.reason;
  *n_out = (int32_t)f.out.size();
  if (out_ids) std::copy(f.out.begin(), f.out.begin() + std::min<size_t>(f.out.size(), (size_t)std::max(cap, 0)), out_ids);
  return SR_OK;
}

static double median_ms(std::vector<double> v) {
  if (v.empty()) return 0.0;
  const size_t k = v.size() / 2;
  std::nth_element(v.begin(), v.begin() + k, v.end());
  double x = v[k];
  if (v.size() % 2 == 0) x = 0.5 * (x + *std::max_element(v.begin(), v.begin() + k));
  return 1000.0 * x;
}

extern "C" int sr_engine_latency(const sr_engine* e, double* ttft_p50_ms, double* itl_p50_ms, int64_t* n_ttft,
                                 int64_t* n_itl) {
  if (!e || !ttft_p50_ms || !itl_p50_ms || !n_ttft || !n_itl) return sr_fail(SR_EINVAL, "null argument");
  *ttft_p50_ms = median_ms(e->ttft);
  *itl_p50_ms = median_ms(e->itl);
  *n_ttft = (int64_t)e->ttft.size();
  *n_itl = (int64_t)e->itl.size();
  return SR_OK;
}

extern "C" int sr_engine_stats_get(const sr_engine* e, sr_engine_stats* s) {
  if (!e || !s) return sr_fail(SR_EINVAL, "null argument");
  *s = e->st;
  s->active = (int64_t)e->sessions.size();
  s->queued = (int64_t)e->queue.size();
  s->pool_limit = e->limit;
  s->pool_reserved = e->reserved;
  s->pool_allocated = e->allocated + e->prefix.pages;
  s->prefix_bytes = (int64_t)e->prefix.pages * e->m->dm.page_elems * 4;
  return SR_OK;
}

extern "C" int sr_engine_last_schedule(const sr_engine* e, int32_t* counts, int32_t cap, int32_t* n_sessions) {
  if (!e || !n_sessions) return sr_fail(SR_EINVAL, "null argument");
  *n_sessions = (int32_t)e->last_counts.size();
  if (counts)
    std::copy(e->last_counts.begin(),
              e->last_counts.begin() + std::min<size_t>(e->last_counts.size(), (size_t)std::max(cap, 0)), counts);
  return SR_OK;
}

extern "C" int sr_engine_session_pages(const sr_engine* e, int32_t i, int32_t* pages, int32_t cap, int32_t* n_pages) {
  if (!e || !n_pages) return sr_fail(SR_EINVAL, "null argument");
  if (i < 0 || i >= (int32_t)e->sessions.size()) return sr_fail(SR_EINVAL, "session index out of range");
  const auto& p = e->sessions[i].pages;
  *n_pages = (int32_t)p.size();
  if (pages) std::copy(p.begin(), p.begin() + std::min<size_t>(p.size(), (size_t)std::max(cap, 0)), pages);
  return SR_OK;
}

extern "C" int sr_engine_set_pieces(sr_engine* e, const uint8_t* pieces, const int64_t* offsets, int32_t vocab,
                                    int32_t flags, const uint8_t* fallback) {
  if (!e || (vocab > 0 && !offsets)) return sr_fail(SR_EINVAL, "null argument");
  if (!e->sessions.empty()) return sr_fail(SR_EINVAL, "token text can be configured only while no session is active");
  if (vocab <= 0) {  // off
    e->text_on = false;
    e->pieces.clear();
    e->piece_off.clear();
    e->fallback.clear();
    return SR_OK;
  }
  if (vocab < e->m->dm.vocab)  // e.pieces[id] must exist for every id the sampler can return
    return sr_fail(SR_EINVAL, "the pieces table must cover the model's vocabulary");
  if (offsets[0] != 0) return sr_fail(SR_EINVAL, "piece offsets must start at 0");
  for (int32_t i = 0; i < vocab; i++)
    if (offsets[i + 1] < offsets[i]) return sr_fail(SR_EINVAL, "piece offsets must not decrease");
  if (offsets[vocab] > 0 && !pieces) return sr_fail(SR_EINVAL, "null pieces");
  sr_text_decoder* probe = nullptr;  // checks the flags and the fallback table
  int rc = sr_text_decoder_create(flags, fallback, (flags & SR_TEXT_MISTRAL) ? vocab : 0, &probe);
  if (rc != SR_OK) return rc;
  sr_text_decoder_destroy(probe);
  e->pieces.assign((const char*)pieces, (size_t)offsets[vocab]);
  e->piece_off.assign(offsets, offsets + vocab + 1);
  e->fallback.clear();
  if ((flags & SR_TEXT_MISTRAL) && fallback) e->fallback.assign(fallback, fallback + vocab);
  e->text_flags = flags;
  e->text_on = true;
  return SR_OK;
}

extern "C" int sr_engine_poll_token(sr_engine* e, int64_t* request_id, int32_t* token_id, char* text, int32_t cap,
                                    int32_t* n_text, int32_t* final) {
  if (!e || !request_id || !token_id || !n_text || !final) return sr_fail(SR_EINVAL, "null argument");
  if (e->events.empty()) {
    *request_id = -1;
    *token_id = -1;
    *n_text = 0;
    *final = 0;
    return SR_OK;
  }
  const TextEvent& ev = e->events.front();
  *n_text = (int32_t)ev.text.size();
  if ((int64_t)ev.text.size() > (int64_t)std::max(cap, 0) || (!text && !ev.text.empty()))
    return sr_fail(SR_EINVAL, "text buffer too small: *n_text bytes needed");  // the event stays queued
  *request_id = ev.request_id;
  *token_id = ev.token_id;
  *final = ev.final;
  if (!ev.text.empty()) memcpy(text, ev.text.data(), ev.text.size());
  e->events.pop_front();
  return SR_OK;
}
