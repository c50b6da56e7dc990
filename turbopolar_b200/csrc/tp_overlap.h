// Host side of the overlap between consecutive decode-attention calls on one stream: the device
// byte ranges a call reads and writes, and whether a call may start streaming its pages before
// the previous call launched on the same stream has completed.  Plain C++ (no CUDA types), so
// the CPU tests compile it on its own.
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>
#include <map>
#include <vector>

namespace tp {

// Device byte range [lo, hi).
struct Span {
  uintptr_t lo, hi;
};

constexpr int kMaxSpans = 12;

// The ranges one call reads, or writes.  More ranges than fit are treated as overlapping
// everything, so an overflow can only make a call wait.
struct Spans {
  Span s[kMaxSpans];
  int n = 0;
  bool all = false;
  void add(const void* p, size_t bytes) {
    if (!p || !bytes) return;
    if (n < kMaxSpans) s[n++] = Span{uintptr_t(p), uintptr_t(p) + bytes};
    else all = true;
  }
  bool meets(const Spans& o) const {
    if (all || o.all) return true;
    for (int i = 0; i < n; ++i)
      for (int j = 0; j < o.n; ++j)
        if (s[i].lo < o.s[j].hi && o.s[j].lo < s[i].hi) return true;
    return false;
  }
};

// The buffers of one attention call (sizes in bytes; NULL pointers are skipped).
struct CallBuffers {
  const void* q = nullptr;             // query, read
  size_t q_bytes = 0;
  const void* pages = nullptr;         // page pool, read (written by a decode step's flush)
  size_t pages_bytes = 0;
  const void* radii_scales = nullptr;  // per-page radius scales, like the pool
  size_t radii_scales_bytes = 0;
  const void* tail_k = nullptr;        // dense tail, read (written by a decode step)
  const void* tail_v = nullptr;
  size_t tail_bytes = 0;               // each of tail_k, tail_v
  const void* d_state = nullptr;       // state words, read (advanced by a decode step)
  size_t state_bytes = 0;
  const void* out = nullptr;           // fp16 output or partials, written
  size_t out_bytes = 0;
  bool step = false;                   // a decode step: appends k_new / v_new first
  const void* k_new = nullptr;         // the new token, read by a decode step
  const void* v_new = nullptr;
  size_t new_bytes = 0;                // each of k_new, v_new
  const void* exchange = nullptr;      // this rank's exchange buffer (sharded call), or NULL
  size_t exchange_bytes = 0;
  const void* values = nullptr;        // dense value array (dense-V call), read
  size_t values_bytes = 0;
  const void* workspace = nullptr;     // partials and error word, written (see StreamLog)
  size_t workspace_bytes = 0;
};

// The workspace of `b`.
inline void workspace_spans(const CallBuffers& b, Spans& out) { out.add(b.workspace, b.workspace_bytes); }

// The cache a page pass reads before griddepcontrol.wait: state words, pages, radius scales.
inline void cache_spans(const CallBuffers& b, Spans& out) {
  out.add(b.d_state, b.state_bytes);
  out.add(b.pages, b.pages_bytes);
  out.add(b.radii_scales, b.radii_scales_bytes);
}

// What `b` reads and writes.  The workspace is left out of both sides (StreamLog tracks it on
// its own): the page pass writes its partials only after griddepcontrol.wait unless no call
// that may still run uses the same workspace, and the split combine reads them after its own.  A
// sharded call's split combine reads and advances the epoch in this rank's exchange buffer
// before its wait, so the buffer counts as read and written and two calls on one exchange
// never overlap (calls on different exchanges, one per layer, may); the other ranks' buffers
// are written only after the wait.
inline void call_spans(const CallBuffers& b, Spans& reads, Spans& writes) {
  reads.add(b.q, b.q_bytes);
  reads.add(b.pages, b.pages_bytes);
  reads.add(b.radii_scales, b.radii_scales_bytes);
  reads.add(b.tail_k, b.tail_bytes);
  reads.add(b.tail_v, b.tail_bytes);
  reads.add(b.d_state, b.state_bytes);
  writes.add(b.out, b.out_bytes);
  if (b.step) {
    reads.add(b.k_new, b.new_bytes);
    reads.add(b.v_new, b.new_bytes);
    writes.add(b.d_state, b.state_bytes);
    writes.add(b.tail_k, b.tail_bytes);
    writes.add(b.tail_v, b.tail_bytes);
    writes.add(b.pages, b.pages_bytes);
    writes.add(b.radii_scales, b.radii_scales_bytes);
  }
  reads.add(b.exchange, b.exchange_bytes);
  writes.add(b.exchange, b.exchange_bytes);
  reads.add(b.values, b.values_bytes);
}

// The writes a new call on a stream must not read early.  Only this library's kernels let a
// dependent grid start before they complete (griddepcontrol.launch_dependents), and any other
// kernel launched between two calls starts after the first has completed; work on other streams
// is ordered by events, which wait for completion.  A call that streams early (independent)
// starts once the previous call's split combine has started, which may be before that call, and
// every independent call before it back to the last call that waited, have completed; so the
// log keeps the union of the writes of every call since (and including) the last one that was
// judged dependent.  A dependent call's page pass waits for its predecessor to complete before
// it lets the next call start, so the union restarts there.  A stream's first call (no entry)
// is judged dependent.
//
// A stream is identified by (device, handle, host thread, capture):
//   - the device, because the legacy default stream (handle 0) and the per-thread default
//     stream are per-device streams behind one handle value;
//   - the host thread for the per-thread default stream handle only, which names a different
//     stream in every host thread;
//   - the id of the stream capture the call is recorded into (0 outside capture).  Inside one
//     capture the recorded order is the replay order, so every decision holds at each replay;
//     the first call of a capture is judged dependent.  A stream records one capture at a time,
//     so entries of its earlier captures are dropped when a new one starts.
struct StreamKey {
  int device;
  uintptr_t stream;
  uint64_t thread;   // 0 unless `stream` is the per-thread default stream handle
  uint64_t capture;  // 0 outside stream capture
  bool operator<(const StreamKey& o) const {
    if (device != o.device) return device < o.device;
    if (stream != o.stream) return stream < o.stream;
    if (thread != o.thread) return thread < o.thread;
    return capture < o.capture;
  }
};

// Writes of a chain of calls.  More ranges than kMaxChain count as overlapping everything, so
// an overflow can only make the next call wait (and restart the chain).
struct ChainWrites {
  static constexpr int kMaxChain = 1024;
  std::vector<Span> s;
  bool all = false;
  void reset(const Spans& w) {
    s.assign(w.s, w.s + w.n);
    all = w.all;
  }
  void add(const Spans& w) {
    if (w.all || s.size() + size_t(w.n) > size_t(kMaxChain)) {
      all = true;
      return;
    }
    s.insert(s.end(), w.s, w.s + w.n);
  }
  bool meets(const Spans& r) const {
    if (all || r.all) return true;
    for (const Span& a : s)
      for (int j = 0; j < r.n; ++j)
        if (a.lo < r.s[j].hi && r.s[j].lo < a.hi) return true;
    return false;
  }
};

// The chain of one stream: its calls' writes and, apart, their workspaces.
struct Chain {
  ChainWrites writes, ws;
};

class StreamLog {
 public:
  // True when this call may read early: the stream has a chain and nothing its calls write is
  // read by this call.  Adds this call's writes to the chain, or restarts the chain with them.
  // With `probe`, *probe_clear tells whether the chain (before this call) writes none of the
  // probe's ranges: what a dependent call reads of them before its wait is then final too.
  // With `ws` (this call's workspace), *ws_clear tells whether the call is independent and no
  // call of the chain uses an overlapping workspace: its page pass may then write its partials
  // before it waits for the previous call (it still waits before it completes, so that its
  // completion implies the previous call's).  The chain keeps the workspaces beside the writes.
  bool independent(const StreamKey& key, const Spans& reads, const Spans& writes, const Spans* probe = nullptr,
                   bool* probe_clear = nullptr, const Spans* ws = nullptr, bool* ws_clear = nullptr) {
    std::lock_guard<std::mutex> lock(mu_);
    const Spans none{};
    const Spans& w = ws ? *ws : none;
    auto it = last_.find(key);
    if (probe_clear) *probe_clear = it != last_.end() && !it->second.writes.meets(*probe);
    if (ws_clear) *ws_clear = false;
    if (it == last_.end()) {
      if (key.capture != 0) {
        for (auto j = last_.begin(); j != last_.end();) {
          const StreamKey& o = j->first;
          if (o.device == key.device && o.stream == key.stream && o.thread == key.thread && o.capture != 0)
            j = last_.erase(j);
          else
            ++j;
        }
      }
      Chain& c = last_[key];
      c.writes.reset(writes);
      c.ws.reset(w);
      return false;
    }
    Chain& c = it->second;
    const bool ok = !c.writes.meets(reads);
    if (ok) {
      if (ws_clear) *ws_clear = !w.all && w.n > 0 && !c.ws.meets(w);
      c.writes.add(writes);
      c.ws.add(w);
    } else {
      c.writes.reset(writes);
      c.ws.reset(w);
    }
    return ok;
  }
  size_t size() {
    std::lock_guard<std::mutex> lock(mu_);
    return last_.size();
  }

 private:
  std::mutex mu_;
  std::map<StreamKey, Chain> last_;
};

}  // namespace tp
