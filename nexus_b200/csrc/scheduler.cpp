// scheduler.cpp -- request scheduler with KV pages, and the continuous-batching
// tick that drives the device with it.
//
// nexus_scheduler_* restates the reference's Scheduler (src/scheduler.rs:
// Request :26-104, ScheduledDecode :106-115, KvPageAllocation :117-124,
// Scheduler :126-361) as host code: FIFO admission up to max_batch_size
// running requests, ceil((prompt_len + max_tokens) / page_size_tokens) KV
// pages per request (at least one) while the pool has them, decode items
// {id, last token, position, generated, prompt_len, kv_pages}, and
// append_generated / step / complete_request moving requests to completed
// and releasing their pages.  One difference: the reference numbers pages
// from a counter that never goes back (the ids are bookkeeping only there);
// here a released id is reused, smallest first, because the ids name real
// pages of the device KV pool (nexus_cuda_seq_set_pages) and must stay below
// max_kv_pages.  Until the first release both give the same ids.
//
// nexus_cuda_serve_step is the serving loop the reference lacks: its server
// takes the engine mutex and runs one generate_with_config per request
// (src/server/mod.rs:407,416), and decode_batch / append_generated are never
// called.  One tick admits pending requests, binds each new request's pages
// to a free device sequence and prefills all but its last prompt token, then
// runs one nexus_cuda_decode_batch step over every running request (the
// scheduler's decode items) and appends each greedy token.  A request's
// tokens therefore equal greedy generate(prompt, max_tokens) on its own.
//
// Position convention: ScheduledDecode.position is the request's token count
// (src/scheduler.rs:94-99: prompt_len, +1 per generated token), so the item's
// token -- the last one -- sits at position - 1 of the sequence; that is the
// position handed to the device step.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <deque>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "../../include/nexus_cuda.h"
#include "trace.h"

namespace {

enum class State { Pending, Running, Done };

struct Request {
    uint64_t id = 0;
    std::vector<uint32_t> tokens;
    State state = State::Pending;
    size_t prompt_len = 0, max_tokens = 0;
    size_t generated = 0, position = 0;  // while Running (RequestState::Running)
    std::vector<uint32_t> kv_pages;
    int seq = -1;                        // device sequence while served

    // Request::advance (src/scheduler.rs:50-70)
    bool advance() {
        if (state != State::Running) return false;
        if (generated >= max_tokens) {
            state = State::Done;
            return false;
        }
        generated++;
        position++;
        if (generated >= max_tokens) state = State::Done;
        return true;
    }
    // Request::generated_tokens / position (:86-103)
    size_t generated_tokens() const {
        if (state == State::Running) return generated;
        if (state == State::Done) return tokens.size() > prompt_len ? tokens.size() - prompt_len : 0;
        return 0;
    }
    size_t pos() const { return state == State::Running ? position : tokens.size(); }
};

}  // namespace

struct nexus_scheduler {
    std::mutex mu;
    size_t max_batch_size = 8, page_size_tokens = 16, max_kv_pages = 0;  // 0 = no limit
    std::deque<Request> pending;
    std::vector<Request> running, completed;
    std::map<uint64_t, size_t> allocations;  // request id -> pages held
    size_t pages_used = 0;
    std::set<uint32_t> released;             // page ids free for reuse
    uint64_t next_page_id = 0;
    std::vector<uint32_t> scratch_pages;     // kv_pages of the last decode_batch call
    // device binding (nexus_cuda_serve_step)
    std::vector<int> free_seqs;              // device sequence ids not serving a request
    bool seqs_ready = false;
    std::vector<int> seqs_to_release;        // sequences of requests that ended outside a tick
};

namespace {

// the calling thread's last scheduler error (nexus_scheduler_last_error)
thread_local std::string g_sched_error;

int fail(const char *msg) {
    g_sched_error = msg;
    return NEXUS_E_INVALID;
}

bool known_id(nexus_scheduler *s, uint64_t id) {
    for (auto &r : s->pending)
        if (r.id == id) return true;
    for (auto &r : s->running)
        if (r.id == id) return true;
    for (auto &r : s->completed)
        if (r.id == id) return true;
    return false;
}

// Scheduler::allocate_kv_pages (src/scheduler.rs:333-361)
bool allocate_pages(nexus_scheduler *s, Request &r) {
    const size_t capacity = r.prompt_len + r.max_tokens;
    const size_t needed = std::max<size_t>(1, (capacity + s->page_size_tokens - 1) / s->page_size_tokens);
    if (s->max_kv_pages && s->pages_used + needed > s->max_kv_pages) return false;
    r.kv_pages.clear();
    for (size_t i = 0; i < needed; i++) {
        if (!s->released.empty()) {
            r.kv_pages.push_back(*s->released.begin());
            s->released.erase(s->released.begin());
        } else {
            r.kv_pages.push_back((uint32_t)s->next_page_id++);
        }
    }
    s->pages_used += needed;
    s->allocations[r.id] = needed;
    return true;
}

// Scheduler::release_kv_pages (:363-365)
void release_pages(nexus_scheduler *s, Request &r) {
    auto it = s->allocations.find(r.id);
    if (it == s->allocations.end()) return;
    s->pages_used -= it->second;
    s->allocations.erase(it);
    for (uint32_t p : r.kv_pages) s->released.insert(p);
}

// A request leaves the running set: its pages go back, its device sequence
// (if any) is handed to the next serve tick for release.
void finish(nexus_scheduler *s, Request &r) {
    release_pages(s, r);
    if (r.seq >= 0) {
        s->seqs_to_release.push_back(r.seq);
        r.seq = -1;
    }
}

// Scheduler::fill_running (:182-204): admitted requests are appended to
// `running`; returns how many.
size_t fill_running(nexus_scheduler *s) {
    size_t admitted = 0;
    const size_t slots = s->max_batch_size > s->running.size() ? s->max_batch_size - s->running.size() : 0;
    while (admitted < slots && !s->pending.empty()) {
        Request r = std::move(s->pending.front());
        s->pending.pop_front();
        if (!allocate_pages(s, r)) {
            s->pending.push_front(std::move(r));
            break;
        }
        // Request::mark_running (:72-79)
        r.state = State::Running;
        r.generated = 0;
        r.position = r.prompt_len;
        s->running.push_back(std::move(r));
        admitted++;
    }
    return admitted;
}

int copy_ids(const std::vector<uint64_t> &v, uint64_t *ids, size_t max, size_t *n) {
    if (n) *n = v.size();
    if (v.size() > max || (v.size() && !ids)) return fail("id buffer too small");
    for (size_t i = 0; i < v.size(); i++) ids[i] = v[i];
    return NEXUS_OK;
}

}  // namespace

extern "C" const char *nexus_scheduler_last_error(void) { return g_sched_error.c_str(); }

extern "C" int nexus_scheduler_create(uint32_t max_batch_size, uint32_t page_size_tokens, uint32_t max_kv_pages,
                                      nexus_scheduler **out) {
    if (!out) return fail("NULL argument");
    *out = nullptr;
    nexus_scheduler *s = new (std::nothrow) nexus_scheduler();
    if (!s) return NEXUS_E_OOM;
    s->max_batch_size = max_batch_size;
    s->page_size_tokens = std::max<uint32_t>(1, page_size_tokens);  // page_size_tokens.max(1), :160
    s->max_kv_pages = max_kv_pages;
    *out = s;
    return NEXUS_OK;
}

extern "C" int nexus_scheduler_destroy(nexus_scheduler *s) {
    delete s;
    return NEXUS_OK;
}

extern "C" int nexus_scheduler_add_request(nexus_scheduler *s, uint64_t id, const uint32_t *tokens, size_t n,
                                           uint32_t max_tokens) {
    if (!s || !tokens) return fail("NULL argument");
    // an empty request would never give a decode item (decode_batch skips it,
    // src/scheduler.rs:217) and would hold its batch slot forever
    if (n == 0) return fail("a request needs at least one token");
    std::lock_guard<std::mutex> lk(s->mu);
    if (known_id(s, id)) return fail("request id already in use");
    Request r;
    r.id = id;
    r.tokens.assign(tokens, tokens + n);
    r.prompt_len = n;
    r.max_tokens = max_tokens;
    s->pending.push_back(std::move(r));
    return NEXUS_OK;
}

extern "C" int nexus_scheduler_get_next_batch(nexus_scheduler *s, uint64_t *ids, size_t max, size_t *n) {
    if (!s) return fail("NULL argument");
    std::lock_guard<std::mutex> lk(s->mu);
    // the ids must fit before anything is admitted
    const size_t slots = s->max_batch_size > s->running.size() ? s->max_batch_size - s->running.size() : 0;
    if (std::min(slots, s->pending.size()) > max) {
        if (n) *n = std::min(slots, s->pending.size());
        return fail("id buffer too small");
    }
    const size_t before = s->running.size();
    fill_running(s);
    std::vector<uint64_t> v;
    for (size_t i = before; i < s->running.size(); i++) v.push_back(s->running[i].id);
    return copy_ids(v, ids, max, n);
}

extern "C" int nexus_scheduler_decode_batch(nexus_scheduler *s, nexus_scheduled_decode *items, size_t max,
                                            size_t *n) {
    if (!s || !n) return fail("NULL argument");
    std::lock_guard<std::mutex> lk(s->mu);
    const size_t slots = s->max_batch_size > s->running.size() ? s->max_batch_size - s->running.size() : 0;
    if (s->running.size() + std::min(slots, s->pending.size()) > max) {
        *n = s->running.size() + std::min(slots, s->pending.size());
        return fail("item buffer too small");
    }
    fill_running(s);
    // Scheduler::decode_batch (:207-229): requests without a token give no item
    size_t total_pages = 0;
    for (auto &r : s->running) total_pages += r.kv_pages.size();
    s->scratch_pages.resize(total_pages);
    size_t k = 0, off = 0;
    for (auto &r : s->running) {
        if (r.tokens.empty()) continue;
        nexus_scheduled_decode &d = items[k++];
        d.id = r.id;
        d.token = r.tokens.back();
        d.position = (uint32_t)r.pos();
        d.generated = (uint32_t)r.generated_tokens();
        d.prompt_len = (uint32_t)r.prompt_len;
        d.n_pages = (uint32_t)r.kv_pages.size();
        std::copy(r.kv_pages.begin(), r.kv_pages.end(), s->scratch_pages.begin() + off);
        d.kv_pages = s->scratch_pages.data() + off;
        off += r.kv_pages.size();
    }
    *n = k;
    return NEXUS_OK;
}

static int append_locked(nexus_scheduler *s, uint64_t id, uint32_t token, int *found) {
    // Scheduler::append_generated (:232-251)
    auto it = std::find_if(s->running.begin(), s->running.end(), [&](const Request &r) { return r.id == id; });
    if (it == s->running.end()) {
        if (found) *found = 0;
        return NEXUS_OK;
    }
    if (it->advance()) it->tokens.push_back(token);
    if (it->state == State::Done) {
        Request r = std::move(*it);
        s->running.erase(it);
        finish(s, r);
        s->completed.push_back(std::move(r));
    }
    if (found) *found = 1;
    return NEXUS_OK;
}

extern "C" int nexus_scheduler_append_generated(nexus_scheduler *s, uint64_t id, uint32_t token, int *found) {
    if (!s) return fail("NULL argument");
    std::lock_guard<std::mutex> lk(s->mu);
    return append_locked(s, id, token, found);
}

extern "C" int nexus_scheduler_step(nexus_scheduler *s, uint64_t *ids, size_t max, size_t *n) {
    if (!s) return fail("NULL argument");
    std::lock_guard<std::mutex> lk(s->mu);
    if (s->running.size() > max) {
        if (n) *n = s->running.size();
        return fail("id buffer too small");
    }
    // Scheduler::step (:254-281)
    std::vector<uint64_t> v;
    for (size_t i = 0; i < s->running.size();) {
        Request &r = s->running[i];
        if (r.state == State::Running && r.advance()) v.push_back(r.id);
        if (r.state == State::Done) {
            Request d = std::move(r);
            s->running.erase(s->running.begin() + (long)i);
            finish(s, d);
            s->completed.push_back(std::move(d));
        } else {
            i++;
        }
    }
    return copy_ids(v, ids, max, n);
}

extern "C" int nexus_scheduler_get_completed(nexus_scheduler *s, uint64_t *ids, size_t max, size_t *n) {
    if (!s) return fail("NULL argument");
    std::lock_guard<std::mutex> lk(s->mu);
    std::vector<uint64_t> v;
    for (auto &r : s->completed) v.push_back(r.id);
    if (v.size() > max) {
        if (n) *n = v.size();
        return fail("id buffer too small");
    }
    // Scheduler::get_completed (:284-287) takes them
    s->completed.clear();
    return copy_ids(v, ids, max, n);
}

extern "C" int nexus_scheduler_complete_request(nexus_scheduler *s, uint64_t id, int *found) {
    if (!s) return fail("NULL argument");
    std::lock_guard<std::mutex> lk(s->mu);
    // Scheduler::complete_request (:290-314)
    if (found) *found = 0;
    for (size_t i = 0; i < s->running.size(); i++) {
        if (s->running[i].id != id) continue;
        Request r = std::move(s->running[i]);
        s->running.erase(s->running.begin() + (long)i);
        r.state = State::Done;
        finish(s, r);
        s->completed.push_back(std::move(r));
        if (found) *found = 1;
        return NEXUS_OK;
    }
    for (size_t i = 0; i < s->pending.size(); i++) {
        if (s->pending[i].id != id) continue;
        Request r = std::move(s->pending[i]);
        s->pending.erase(s->pending.begin() + (long)i);
        r.state = State::Done;
        finish(s, r);
        s->completed.push_back(std::move(r));
        if (found) *found = 1;
        return NEXUS_OK;
    }
    return NEXUS_OK;
}

extern "C" int nexus_scheduler_stats(nexus_scheduler *s, size_t *pending, size_t *running, size_t *completed) {
    if (!s) return fail("NULL argument");
    std::lock_guard<std::mutex> lk(s->mu);
    if (pending) *pending = s->pending.size();
    if (running) *running = s->running.size();
    if (completed) *completed = s->completed.size();
    return NEXUS_OK;
}

extern "C" int nexus_scheduler_kv_page_stats(nexus_scheduler *s, size_t *used, size_t *max_pages) {
    if (!s) return fail("NULL argument");
    std::lock_guard<std::mutex> lk(s->mu);
    if (used) *used = s->pages_used;
    if (max_pages) *max_pages = s->max_kv_pages;
    return NEXUS_OK;
}

extern "C" int nexus_scheduler_kv_allocation(nexus_scheduler *s, uint64_t id, uint32_t *page_ids, size_t max,
                                             size_t *n, size_t *capacity_tokens) {
    if (!s || !n) return fail("NULL argument");
    std::lock_guard<std::mutex> lk(s->mu);
    *n = 0;
    if (!s->allocations.count(id)) return fail("the request holds no KV pages");  // kv_allocation -> None
    for (auto &r : s->running) {
        if (r.id != id) continue;
        *n = r.kv_pages.size();
        if (capacity_tokens) *capacity_tokens = r.prompt_len + r.max_tokens;
        if (r.kv_pages.size() > max || (r.kv_pages.size() && !page_ids)) return fail("page buffer too small");
        std::copy(r.kv_pages.begin(), r.kv_pages.end(), page_ids);
        return NEXUS_OK;
    }
    return NEXUS_E_INVALID;
}

extern "C" int nexus_scheduler_tokens(nexus_scheduler *s, uint64_t id, uint32_t *out, size_t max, size_t *n) {
    if (!s || !n) return fail("NULL argument");
    std::lock_guard<std::mutex> lk(s->mu);
    auto emit = [&](const Request &r) {
        *n = r.tokens.size();
        if (r.tokens.size() > max || (r.tokens.size() && !out)) return fail("token buffer too small");
        std::copy(r.tokens.begin(), r.tokens.end(), out);
        return (int)NEXUS_OK;
    };
    for (auto &r : s->running)
        if (r.id == id) return emit(r);
    for (auto &r : s->completed)
        if (r.id == id) return emit(r);
    for (auto &r : s->pending)
        if (r.id == id) return emit(r);
    *n = 0;
    return fail("unknown request id (completed requests are forgotten once taken)");
}

// ---------------------------------------------------------------------------
// Continuous batching on the device.

extern "C" int nexus_cuda_serve_step(nexus_cuda_model *m, nexus_scheduler *s, nexus_serve_event *events,
                                     size_t max_events, size_t *n_events) {
    nx::TraceRange tr("nexus_cuda_serve_step");
    g_sched_error.clear();  // a failure below names itself here or in the backend's last error
    if (!m || !s || !n_events) return fail("NULL argument");
    *n_events = 0;
    nexus_cuda_model_info info = {};
    int rc = nexus_cuda_model_get_info(m, &info);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(s->mu);
    if (s->page_size_tokens != info.page_tokens) return fail("scheduler page size differs from the model's KV pages");
    if (s->max_kv_pages == 0 || s->max_kv_pages > info.max_pages)
        return fail("max_kv_pages must be set and within the model's KV page pool");
    if (s->max_batch_size > info.max_batch) return fail("max_batch_size above the model's max_batch");
    if (s->max_batch_size > max_events) return fail("event buffer smaller than max_batch_size");
    if (!s->seqs_ready) {
        // the scheduler owns every sequence of the model from here on: pages
        // a sequence held before (the library's default ones) go back to the pool
        for (int q = (int)info.max_batch - 1; q >= 0; q--) {
            rc = nexus_cuda_seq_set_pages(m, (uint32_t)q, nullptr, 0);
            if (rc) return rc;
            s->free_seqs.push_back(q);
        }
        s->seqs_ready = true;
    }
    // sequences of requests completed or cancelled since the last tick
    for (int q : s->seqs_to_release) {
        rc = nexus_cuda_seq_set_pages(m, (uint32_t)q, nullptr, 0);
        if (rc) return rc;
        s->free_seqs.push_back(q);
    }
    s->seqs_to_release.clear();

    // admission: pages bound to a free device sequence, prompt prefilled up
    // to its last token (which the decode step below consumes)
    const size_t before = s->running.size();
    // fill_running, except that a request the model cannot hold (its prompt
    // and max_tokens beyond max_seq_len) ends at once with an error event; it
    // takes an admission slot, so a tick never reports more than
    // max_batch_size events
    for (size_t slots = s->max_batch_size - s->running.size(); slots > 0 && !s->pending.empty(); slots--) {
        Request &front = s->pending.front();
        if (front.prompt_len + front.max_tokens > (size_t)info.max_seq_len + 1) {
            Request d = std::move(front);
            s->pending.pop_front();
            d.state = State::Done;
            events[(*n_events)++] = {d.id, 0, 0, 1, NEXUS_E_INVALID};
            s->completed.push_back(std::move(d));
            continue;
        }
        Request r = std::move(front);
        s->pending.pop_front();
        if (!allocate_pages(s, r)) {
            s->pending.push_front(std::move(r));
            break;
        }
        r.state = State::Running;
        r.generated = 0;
        r.position = r.prompt_len;
        s->running.push_back(std::move(r));
    }
    const uint32_t per_seq = (info.max_seq_len + info.page_tokens - 1) / info.page_tokens;
    // New requests: one with nothing to generate finishes here (Request::advance
    // on generated >= max_tokens, src/scheduler.rs:50-70) without a sequence;
    // the others get a device sequence with their pages bound and their prompt
    // prefilled up to its last token.  A request whose set-up fails ends with
    // an error event (the failing call's status; its message stays in the
    // backend's last error) and gives its sequence and pages back.
    std::vector<uint64_t> zero;
    std::vector<std::pair<uint64_t, int>> broken;
    for (size_t i = before; i < s->running.size(); i++) {
        Request &r = s->running[i];
        if (r.max_tokens == 0) {
            zero.push_back(r.id);
            continue;
        }
        r.seq = s->free_seqs.back();
        s->free_seqs.pop_back();
        const uint32_t np = (uint32_t)std::min<size_t>(r.kv_pages.size(), per_seq);
        rc = nexus_cuda_seq_set_pages(m, (uint32_t)r.seq, r.kv_pages.data(), np);
        if (!rc) rc = nexus_cuda_prefill(m, (uint32_t)r.seq, r.tokens.data(), r.prompt_len - 1, nullptr, nullptr);
        if (rc) broken.push_back({r.id, rc});
    }
    for (uint64_t id : zero) {
        append_locked(s, id, 0, nullptr);
        events[(*n_events)++] = {id, 0, 0, 1, 0};
    }
    for (const auto &b : broken) {
        auto it = std::find_if(s->running.begin(), s->running.end(), [&](const Request &r) { return r.id == b.first; });
        Request r = std::move(*it);
        s->running.erase(it);
        r.state = State::Done;
        finish(s, r);
        s->completed.push_back(std::move(r));
        events[(*n_events)++] = {b.first, 0, 0, 1, b.second};
    }
    for (int q : s->seqs_to_release) {
        rc = nexus_cuda_seq_set_pages(m, (uint32_t)q, nullptr, 0);
        if (rc) return rc;
        s->free_seqs.push_back(q);
    }
    s->seqs_to_release.clear();
    if (s->running.empty()) return NEXUS_OK;

    // one decode step over every running request (Scheduler::decode_batch items)
    std::vector<nexus_decode_item> items;
    std::vector<uint64_t> ids;
    for (auto &r : s->running) {
        nexus_decode_item d = {};
        d.seq_id = (uint32_t)r.seq;
        d.token = r.tokens.back();
        d.position = (uint32_t)(r.pos() - 1);
        items.push_back(d);
        ids.push_back(r.id);
    }
    std::vector<uint32_t> toks(items.size());
    rc = nexus_cuda_decode_batch(m, items.data(), items.size(), toks.data(), nullptr);
    if (rc) return rc;
    for (size_t i = 0; i < ids.size(); i++) {
        auto it = std::find_if(s->running.begin(), s->running.end(), [&](const Request &r) { return r.id == ids[i]; });
        const uint32_t index = (uint32_t)it->generated;
        append_locked(s, ids[i], toks[i], nullptr);
        const bool done = std::none_of(s->running.begin(), s->running.end(),
                                       [&](const Request &r) { return r.id == ids[i]; });
        events[(*n_events)++] = {ids[i], toks[i], index, done ? 1u : 0u, 0};
    }
    for (int q : s->seqs_to_release) {
        rc = nexus_cuda_seq_set_pages(m, (uint32_t)q, nullptr, 0);
        if (rc) return rc;
        s->free_seqs.push_back(q);
    }
    s->seqs_to_release.clear();
    return NEXUS_OK;
}
